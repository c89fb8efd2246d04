"""CPU statement of the expert-parallel loop's compute steps (test infrastructure).

Lets the exchange logic of spider_web_moe_b200.ep (capacity packing, ownership,
all-to-all layouts, combine) run on CPU ranks with the gloo backend.  The
routing, messages, expert FFN and epilogue come from the oracle; the packing is
the layout sb_ep_pack documents: owner q's rows are the tokens that routed to
one of q's experts, ascending, with q's local expert id per slot (-1 otherwise),
and ret_pos marks the first slot of each owner.
"""
import torch

from oracle import spider_oracle as O


class CpuOps:
    def __init__(self, p: O.BlockParams, cfg, rank: int, world: int):
        self.p, self.cfg, self.rank, self.world = p, cfg, rank, world

    def route(self, h, loop_idx):
        cfg, p = self.cfg, self.p
        top_w, top_idx, _ = O.router(h, p.router_w, p.loop_bias[loop_idx], cfg.top_k)
        eidx, ew, _ = O.edge_graph(h, p.loop_emb[loop_idx], p.gen_w, p.gen_b, cfg.num_experts, cfg.edges_per_expert)
        coef = O.destination_coefficients(top_idx, eidx, ew, cfg.num_experts)
        return O.messages_from_coefficients(h, p.edge_w, coef), top_idx.int(), top_w

    def pack(self, top_idx, top_w, msgs, cap):
        n, K = top_idx.shape
        W, H = self.world, msgs.shape[1]
        send_x = torch.zeros(W, cap, H)
        send_idx = torch.full((W, cap, K), -1, dtype=torch.int32)
        send_w = torch.zeros(W, cap, K)
        ret_pos = torch.full((n, K), -1, dtype=torch.int32)
        count = [0] * W
        for t in range(n):
            seen = set()
            for k in range(K):
                q = int(top_idx[t, k]) % W
                if q in seen:
                    continue
                seen.add(q)
                j = count[q]
                count[q] += 1
                send_x[q, j] = msgs[t]
                for kk in range(K):
                    e = int(top_idx[t, kk])
                    send_idx[q, j, kk] = e // W if e % W == q else -1
                    send_w[q, j, kk] = top_w[t, kk]
                ret_pos[t, k] = q * cap + j
        # one packed fp32 tensor per row: [message | ids | weights], as the device layout
        packed = torch.cat([send_x, send_idx.float(), send_w], dim=-1)
        return packed, ret_pos

    def experts(self, packed):
        p = self.p
        K = self.cfg.top_k
        H = packed.shape[-1] - 2 * K
        rows, ids, weights = packed[..., :H], packed[..., H:H + K].long(), packed[..., H + K:]
        W, cap, _ = rows.shape
        out = torch.zeros(W, cap, H)
        for q in range(W):
            for j in range(cap):
                for k in range(ids.shape[-1]):
                    lid = int(ids[q, j, k])
                    if lid < 0:
                        continue
                    e = self.rank + self.world * lid
                    y = O.expert_ffn(rows[q, j:j + 1], p.w_up[e], p.b_up[e], p.w_down[e], p.b_down[e])
                    out[q, j] += weights[q, j, k] * y[0]
        return out

    def epilogue(self, ret, ret_pos, h, x0):
        flat = ret.reshape(-1, ret.shape[-1])
        delta = torch.zeros_like(h)
        for t in range(h.shape[0]):
            for k in range(ret_pos.shape[1]):
                r = int(ret_pos[t, k])
                if r >= 0:
                    delta[t] += flat[r]
        return O.block_epilogue(h, delta, x0, self.p.ln_w, self.p.ln_b, self.cfg.residual_scale,
                                self.cfg.re_inject_weight)
