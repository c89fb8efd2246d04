"""sb_group on the GPU vs the dispatch-plan semantics, bit-exact, at sizes that take
both the single-CTA path (<= 2048 entries) and the multi-CTA path.

The CPU statement below is build_dispatch_plan (spider_infer/forge/ep/
dispatch.py:56-115) generalised to `slots` entries per row: groups ascending,
rows ascending inside a group, a repeated id in a row merged into its first
slot with the weights summed, entries with summed weight <= 0 dropped when
SB_GROUP_POSITIVE_ONLY is set, ids outside [0, G) skipped.
"""
import pytest
import torch

from spider_web_moe_b200 import _lib as L

pytestmark = pytest.mark.gpu


def cpu_grouping(idx, w, G, positive_only):
    n, slots = idx.shape
    per_group = [[] for _ in range(G)]
    inv = torch.full((n * slots,), -1, dtype=torch.int32)
    for r in range(n):
        row = idx[r].tolist()
        for s, g in enumerate(row):
            if g < 0 or g >= G or g in row[:s]:
                continue
            wsum = float(sum(w[r, j] for j in range(slots) if row[j] == g)) if w is not None else float(row.count(g))
            if positive_only and not wsum > 0:
                continue
            per_group[g].append((r, r * slots + s, wsum))
    offsets = [0]
    rows, slot_ids, ws = [], [], []
    for g in range(G):
        for (r, e, wsum) in per_group[g]:
            inv[e] = len(rows)
            rows.append(r)
            slot_ids.append(e)
            ws.append(wsum)
        offsets.append(len(rows))
    return (torch.tensor(offsets, dtype=torch.int32), torch.tensor(rows, dtype=torch.int32),
            torch.tensor(slot_ids, dtype=torch.int32), torch.tensor(ws, dtype=torch.float32), inv)


@pytest.mark.parametrize("n_rows,slots,G,positive", [(50, 2, 16, True), (700, 3, 7, False), (3000, 4, 64, True),
                                                     (12000, 8, 128, False), (40000, 2, 16, True)])
def test_group_matches_dispatch_plan(n_rows, slots, G, positive, cuda_device):
    lib = L.load()
    g = torch.Generator().manual_seed(n_rows + slots)
    idx = torch.randint(-1, G, (n_rows, slots), generator=g, dtype=torch.int32)
    idx[::5, -1] = idx[::5, 0]                    # repeated ids inside a row
    w = (torch.rand(n_rows, slots, generator=g) - 0.05).float()
    w32 = w.clone()
    # the summed weights are compared exactly: sum in slot order as the kernel does
    want = cpu_grouping(idx, w32, G, positive)
    d_idx, d_w = idx.to(cuda_device), w.to(cuda_device)
    cap = n_rows * slots
    out = {k: torch.full((cap,), -9, dtype=torch.int32, device=cuda_device) for k in ("row", "slot", "inv")}
    perm_w = torch.zeros(cap, device=cuda_device)
    offsets = torch.zeros(G + 1, dtype=torch.int32, device=cuda_device)
    ws = torch.zeros(lib.sb_group_workspace_bytes(n_rows, slots, G), dtype=torch.uint8, device=cuda_device)
    for _ in range(2):  # twice: the workspace's counters must be left ready for the next call
        rc = lib.sb_group(d_idx.data_ptr(), d_w.data_ptr(), n_rows, slots, G,
                          L.SB_GROUP_POSITIVE_ONLY if positive else 0, offsets.data_ptr(), out["row"].data_ptr(),
                          out["slot"].data_ptr(), perm_w.data_ptr(), out["inv"].data_ptr(), ws.data_ptr(),
                          ws.numel(), torch.cuda.current_stream().cuda_stream)
        L.check(rc, "sb_group")
        torch.cuda.synchronize()
        off, rows, slot_ids, wsum, inv = want
        used = int(off[-1])
        assert torch.equal(offsets.cpu(), off)
        assert torch.equal(out["row"].cpu()[:used], rows)
        assert torch.equal(out["slot"].cpu()[:used], slot_ids)
        assert torch.equal(out["inv"].cpu(), inv)
        assert torch.allclose(perm_w.cpu()[:used], wsum, rtol=1e-6, atol=1e-7)
