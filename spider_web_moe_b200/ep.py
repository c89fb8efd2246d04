"""Token-sharded expert parallelism for the recurrent Spider-MoE block.

Every rank holds its own batch of tokens and the block's dense weights
(router, edge generator, edge values, LayerNorm); the experts are sharded the
reference's way, rank ``r`` owning the experts ``e % world == r``
(spider_moe/expert_parallel.py:29-30).  One loop on a rank:

1. route: router, edge graph and messages of its own tokens (sb_block_route);
2. pack: each token's message row once per owner of one of its experts, into a
   fixed-capacity buffer [world, cap] of packed rows (message, the owner's local
   expert ids, routing weights; sb_ep_pack; cap = the agreed tokens per rank,
   so no host round trip is needed to size the exchange);
3. all-to-all of the packed rows (NCCL over NVLink);
4. experts: the owner runs its local experts on the received rows and sums
   each row's weighted outputs (sb_expert_rows);
5. all-to-all back;
6. epilogue: per token, the sum of the rows returned by its owners is the
   expert delta, then LayerNorm(h + 0.5 delta + 0.1 x0) (sb_combine_ln).

The reference instead replicates all tokens on every rank and all-reduces the
full delta (expert_parallel.py:33-37); ``SpiderMoELayer`` keeps that contract,
this module is the sharded path measured by ``bench.py --gpus N``.

The loop is written against an ``ops`` object (route / pack / experts /
epilogue) so that the exchange logic itself can be checked on CPU ranks with
the gloo backend; ``CudaOps`` is the implementation that runs the kernels.
"""
from __future__ import annotations

import ctypes as C
import dataclasses

import torch
import torch.distributed as dist

from . import _lib as L
from .config import from_any
from .engine import BlockEngine


def local_expert_ids(num_experts: int, rank: int, world: int) -> list[int]:
    return [e for e in range(num_experts) if e % world == rank]


def local_expert_state(state: dict, num_experts: int, rank: int, world: int) -> dict:
    """The rank's experts renamed to local ids j (global id rank + world*j)."""
    out = {}
    for j, e in enumerate(local_expert_ids(num_experts, rank, world)):
        for pre in ("experts", "expert_gates"):
            for k, v in state.items():
                head = f"{pre}.{e}."
                if k.startswith(head):
                    out[f"{pre}.{j}." + k[len(head):]] = v
    return out


class CudaOps:
    """The EP loop's compute steps on one GPU (libspider_b200)."""

    def __init__(self, dense: BlockEngine, local: BlockEngine | None, world: int):
        self.dense, self.local, self.world = dense, local, world

    def route(self, h, loop_idx):
        return self.dense.route(h, loop_idx)

    def pack(self, top_idx, top_w, msgs, cap):
        return self.dense.ep_pack(top_idx, top_w, msgs, self.world, cap)

    def experts(self, rows):
        W, cap, pitch = rows.shape
        H = self.dense.cfg.hidden_size
        if self.local is None:
            return torch.zeros(W, cap, H, dtype=torch.float32, device=rows.device)
        # each source rank sends on average cap*K/world (row, expert) pairs per owner
        expected = cap * self.dense.cfg.top_k
        return self.local.expert_rows(rows.view(W * cap, pitch), expected_pairs=expected).view(W, cap, H)

    def epilogue(self, ret, ret_pos, h, x0):
        return self.dense.epilogue(ret.reshape(-1, ret.shape[-1]), ret_pos, h, x0)


def ep_loop(ops, h, x0, loop_idx: int, world: int, cap: int, group=None):
    """One loop of the token-sharded block on this rank (see the module docstring).
    Two collectives: the packed dispatch rows out, the owners' combined rows back."""
    msgs, top_idx, top_w = ops.route(h, loop_idx)
    send, ret_pos = ops.pack(top_idx, top_w, msgs, cap)
    if world > 1:
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)
    else:
        recv = send
    rows = ops.experts(recv)
    if world > 1:
        ret = torch.empty_like(rows)
        dist.all_to_all_single(ret, rows, group=group)
    else:
        ret = rows
    return ops.epilogue(ret, ret_pos, h, x0)


class _DeviceBuffer:
    """A raw device allocation seen by torch.as_tensor (no copy, no ownership)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerExchange:
    """Exchange regions of the peer-memory transport (sb_ep_peer_*): this rank's
    region is created here and every other rank's mapped through CUDA IPC, over
    NVLink on one node.  Set-up only; the per-step calls only read and write the
    regions.  Every rank must construct it (the IPC handles are all-gathered)."""

    def __init__(self, world: int, rank: int, cap: int, pitch: int, hidden: int, device, group=None):
        self.lib = L.load()
        self.world, self.rank, self.cap, self.pitch, self.hidden = world, rank, cap, pitch, hidden
        region = C.c_void_p()
        handle = (C.c_uint8 * 64)()
        L.check(self.lib.sb_ep_peer_create(world, cap, pitch, hidden, C.byref(region), handle), "sb_ep_peer_create")
        self.region = int(region.value)
        handles = [bytes(handle)]
        if world > 1:
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
            gathered = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(gathered, mine, group=group)
            handles = [bytes(t.cpu().tolist()) for t in gathered]
        ptrs, self.mapped = [], []
        for q in range(world):
            if q == rank:
                ptrs.append(self.region)
                continue
            p = C.c_void_p()
            buf = (C.c_uint8 * 64).from_buffer_copy(handles[q])
            L.check(self.lib.sb_ep_peer_map(buf, C.byref(p)), "sb_ep_peer_map")
            ptrs.append(int(p.value))
            self.mapped.append(int(p.value))
        self.regions = torch.tensor(ptrs, dtype=torch.int64, device=device)
        ret_off = (world * cap * pitch + 255) // 256 * 256
        self.recv = torch.as_tensor(_DeviceBuffer(self.region, (world, cap, pitch), "|u1"), device=device)
        self.ret = torch.as_tensor(_DeviceBuffer(self.region + ret_off, (world * cap, hidden), "<f4"), device=device)
        self.out = torch.zeros((world * cap, hidden), dtype=torch.float32, device=device)

    def close(self, group=None):
        """Unmap the peers' regions and free this rank's (all ranks, after the
        last step; before the process group is destroyed)."""
        torch.cuda.synchronize()
        if self.world > 1 and dist.is_initialized():
            dist.barrier(group=group)
        for p in self.mapped:
            self.lib.sb_ep_peer_unmap(C.c_void_p(p))
        self.mapped = []
        if self.world > 1 and dist.is_initialized():
            dist.barrier(group=group)
        if self.region:
            self.recv = self.ret = None
            self.lib.sb_ep_peer_destroy(C.c_void_p(self.region))
            self.region = 0


def ep_loop_peer(dense: BlockEngine, local: BlockEngine | None, xch: PeerExchange, h, x0, loop_idx: int,
                 expected_pairs: int, stream=None):
    """One loop of the token-sharded block over the peer-memory transport:
    route -> dispatch into the owners' regions -> (owner) wait, local experts
    on the received rows, results into the sources' regions -> (source) wait,
    epilogue.  The waits run inside the owner's first and the epilogue kernel."""
    lib = xch.lib
    W, cap, pitch, H = xch.world, xch.cap, xch.pitch, xch.hidden
    sp = torch.cuda.current_stream().cuda_stream if stream is None else stream.cuda_stream
    msgs, top_idx, top_w = dense.route(h, loop_idx)
    ret_pos = dense.ep_dispatch(top_idx, top_w, msgs, W, xch.rank, cap, xch.regions)
    if local is not None:
        local.expert_rows_peer(xch, expected_pairs, dense.status_ptr())
    else:
        # no local experts: still take part in the exchange (zero rows back)
        L.check(lib.sb_ep_wait(C.c_void_p(xch.region), W, cap, pitch, H, 0, C.c_void_p(dense.status_ptr()),
                               C.c_void_p(sp)), "sb_ep_wait")
        L.check(lib.sb_ep_return(C.c_void_p(xch.out.data_ptr()), W, xch.rank, cap, pitch, H,
                                 C.c_void_p(xch.regions.data_ptr()), C.c_void_p(sp)), "sb_ep_return")
    return dense.ep_epilogue_peer(xch, ret_pos, h, x0)


class _MicroBatch:
    """One micro-batch of the token-sharded step: engines with workspaces of
    their own (the weights are shared), its own exchange group, stream and,
    with the peer transport, its own exchange regions."""

    def __init__(self, dense, local, group, stream, xch, world):
        self.dense, self.local, self.group, self.stream, self.xch = dense, local, group, stream, xch
        self.ops = CudaOps(dense, local, world)


class ExpertParallelBlock:
    """The block on one rank of a token-sharded expert-parallel group.

    ``micro_batches=2`` splits every rank's tokens into two halves that run
    all loops on two streams with their own exchange groups (NCCL
    communicators, or peer regions): one half's dispatch / return exchange
    overlaps the other half's routing and expert GEMMs.  The block is
    token-independent, so the halves need no exchange of their own.  Every
    rank must use the same setting (the groups are created collectively)."""

    def __init__(self, cfg, state: dict, device, group=None, act_dtype=torch.bfloat16, max_tokens: int = 64,
                 weight_format: str | None = None, engine: str = "auto", transport: str = "nccl",
                 micro_batches: int = 1):
        self.cfg = from_any(cfg)
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if micro_batches not in (1, 2):
            raise ValueError(f"micro_batches={micro_batches}: 1 or 2")
        if transport not in ("nccl", "peer"):
            raise ValueError(f"transport {transport!r}: 'nccl' or 'peer'")
        self.micro_batches, self.transport, self.max_tokens = int(micro_batches), transport, int(max_tokens)
        E = self.cfg.num_experts
        dense_state = {k: v for k, v in state.items() if not k.startswith(("experts.", "expert_gates."))}
        self.dense = BlockEngine(self.cfg, dense_state, device, act_dtype=act_dtype, max_tokens=max_tokens,
                                 weight_format="bf16" if act_dtype == torch.bfloat16 else "native", engine=engine)
        ids = local_expert_ids(E, self.rank, self.world)
        self.local = None
        if ids:
            lcfg = dataclasses.replace(self.cfg, num_experts=len(ids))
            # an owner receiving prefill-size exchanges (>= 128 expected rows per
            # local expert) keeps fp8 / int4 experts resident as bf16 copies
            rows_per_expert = max_tokens * self.world * self.cfg.top_k // max(1, E)
            self.local = BlockEngine(lcfg, local_expert_state(state, E, self.rank, self.world), device,
                                     act_dtype=act_dtype, max_tokens=1, weight_format=weight_format, engine=engine,
                                     resident_bf16=act_dtype == torch.bfloat16 and rows_per_expert >= 128)
        # exchange capacity per micro-batch: its share of max_tokens on every rank
        self.cap = -(-self.max_tokens // self.micro_batches)
        pitch = None
        if transport == "peer":
            # every rank's own dense engine workspace exists before the first step
            self.dense._ensure_workspace(max_tokens)
            pitch = self.dense.lib.sb_ep_row_pitch(self.cfg.hidden_size, self.dense.dims.act_dtype, self.cfg.top_k)
        ranks = dist.get_process_group_ranks(group) if (group is not None and dist.is_initialized()) else \
            list(range(self.world))
        self.mbs = []
        for i in range(self.micro_batches):
            dense = self.dense if i == 0 else self.dense.twin()
            local = self.local if (i == 0 or self.local is None) else self.local.twin()
            g = group if i == 0 else (dist.new_group(ranks=ranks) if self.world > 1 else None)
            stream = None if self.micro_batches == 1 else torch.cuda.Stream(device=device)
            xch = None
            if transport == "peer":
                xch = PeerExchange(self.world, self.rank, self.cap, pitch, self.cfg.hidden_size, device, g)
            self.mbs.append(_MicroBatch(dense, local, g, stream, xch, self.world))
        self.ops, self.xch = self.mbs[0].ops, self.mbs[0].xch

    def _loop_mb(self, mb: _MicroBatch, h, x0, loop_idx: int):
        if self.transport == "peer":
            return ep_loop_peer(mb.dense, mb.local, mb.xch, h, x0, loop_idx, self.cap * self.cfg.top_k,
                                stream=mb.stream)
        return ep_loop(mb.ops, h, x0, loop_idx, self.world, self.cap, mb.group)

    def loop(self, h, x0, loop_idx: int):
        """One loop; every rank must call it (the exchange is collective).  The
        exchange capacity is max_tokens on every rank, so ranks may hold
        different token counts up to that."""
        return self.forward(h, x0, loop_idx, loop_idx + 1)

    def forward(self, h, x0, loop_begin: int = 0, loop_end: int | None = None):
        loop_end = self.cfg.num_loops if loop_end is None else loop_end
        H = self.cfg.hidden_size
        n = h.numel() // H
        if n > self.max_tokens:
            raise ValueError(f"{n} tokens exceed max_tokens={self.max_tokens} of the expert-parallel block")
        h2, x2 = h.reshape(n, H), x0.reshape(n, H)
        if self.micro_batches == 1:
            for l in range(loop_begin, loop_end):
                h2 = self._loop_mb(self.mbs[0], h2, x2, l)
            return h2.view(h.shape)
        if n < self.micro_batches:
            raise ValueError(f"{n} tokens: micro_batches={self.micro_batches} needs at least that many per rank")
        n0 = -(-n // 2)
        cur = torch.cuda.current_stream(h.device)
        parts = [(h2[:n0], x2[:n0]), (h2[n0:], x2[n0:])]
        outs = []
        for mb, (hp, xp) in zip(self.mbs, parts):
            mb.stream.wait_stream(cur)
            hp.record_stream(mb.stream)
            xp.record_stream(mb.stream)
            outs.append(hp)
        # enqueue the halves loop by loop so both streams always hold work
        for l in range(loop_begin, loop_end):
            for i, mb in enumerate(self.mbs):
                with torch.cuda.stream(mb.stream):
                    outs[i] = self._loop_mb(mb, outs[i], parts[i][1], l)
        for mb, o in zip(self.mbs, outs):
            cur.wait_stream(mb.stream)
            o.record_stream(cur)
        return torch.cat(outs).view(h.shape)

    def check_status(self):
        for mb in self.mbs:
            mb.dense.check_status()

    # ------------------------------------------------------------------ CUDA graph
    def capture(self, n_tokens: int):
        """Capture all loops (kernels and the NCCL exchanges) of one step for a fixed
        token count in one CUDA graph.  Every rank must call it.  Release the graph
        (``release_graph``) before destroying the process group."""
        H = self.cfg.hidden_size
        dev = self.dense.device
        dt = self.dense.act_dtype
        self.g_h = torch.zeros(n_tokens, H, dtype=dt, device=dev)
        self.g_x0 = torch.zeros(n_tokens, H, dtype=dt, device=dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):  # sizes every workspace and warms the communicator up
                self.g_out = self.forward(self.g_h, self.g_x0)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        lib = L.load()
        before = lib.sb_kernel_launches()
        with torch.cuda.graph(self.graph):
            self.g_out = self.forward(self.g_h, self.g_x0)
        self.kernels_per_replay = int(lib.sb_kernel_launches() - before)  # library kernels (NCCL not counted)
        torch.cuda.synchronize(dev)

    def replay(self, h=None, x0=None):
        if h is not None:
            self.g_h.copy_(h.reshape(self.g_h.shape), non_blocking=True)
        if x0 is not None:
            self.g_x0.copy_(x0.reshape(self.g_x0.shape), non_blocking=True)
        self.graph.replay()
        return self.g_out

    def release_graph(self):
        self.graph = None

    def close(self):
        """Release the peer-memory exchanges (all ranks; before the process group
        is destroyed)."""
        self.release_graph()
        for mb in self.mbs:
            if mb.xch is not None:
                mb.xch.close(mb.group)
                mb.xch = None
        self.xch = None

