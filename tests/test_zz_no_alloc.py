"""sb_group_noalloc: the grouping entry point that allocates nothing.

Some callers cannot allocate device memory -- a thin binding that only passes
on pointers it was given, or a process whose device memory another allocator's
pool has reserved -- so they cannot supply the workspace sb_group needs.
sb_group_noalloc keeps its scratch in a fixed device array inside the library
instead.  This test calls it through the C ABI twice in a row (different
inputs, so the second call runs over the first call's leftovers in the shared
array) and checks each result against sb_group with a caller workspace.  At
these sizes the two are different kernels (sb_group takes its multi-CTA
two-pass path, sb_group_noalloc the single-CTA one), but both sum a token's
weights in slot order in the same helper, so the permutation (integer work)
and the summed weights must both match exactly.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one; it also passes alone in a fresh process.
"""
import ctypes as C

import pytest
import torch

from spider_web_moe_b200 import _lib as L

pytestmark = pytest.mark.gpu

MAX_ENTRIES = 65536  # SB_GROUP_NOALLOC_MAX_ENTRIES in include/spider_b200.h


def make_entries(n_rows, slots, groups, seed, device):
    g = torch.Generator(device="cpu").manual_seed(seed)
    idx = torch.randint(-1, groups, (n_rows, slots), generator=g, dtype=torch.int32)
    # repeated ids inside a row (merged into the first slot) and non-positive weights (dropped)
    idx[::7, -1] = idx[::7, 0]
    w = torch.rand(n_rows, slots, generator=g) - 0.1
    return idx.to(device), w.to(device)


def outputs(n_rows, slots, groups, device):
    cap = n_rows * slots
    z = lambda n, dt: torch.full((n,), -7, dtype=dt, device=device)  # noqa: E731
    return dict(offsets=z(groups + 1, torch.int32), perm_row=z(cap, torch.int32), perm_slot=z(cap, torch.int32),
                perm_w=torch.full((cap,), float("nan"), device=device), inv=z(cap, torch.int32))


def call(fn_name, idx, w, n_rows, slots, groups, flags, out, ws=None):
    lib = L.load()
    stream = torch.cuda.current_stream().cuda_stream
    args = [idx.data_ptr(), w.data_ptr(), n_rows, slots, groups, flags, out["offsets"].data_ptr(),
            out["perm_row"].data_ptr(), out["perm_slot"].data_ptr(), out["perm_w"].data_ptr(), out["inv"].data_ptr()]
    if fn_name == "sb_group":
        rc = lib.sb_group(*args, ws.data_ptr(), ws.numel(), stream)
    else:
        rc = lib.sb_group_noalloc(*args, stream)
    L.check(rc, fn_name)


def test_noalloc_grouping_matches_workspace_grouping_twice(cuda_device):
    lib = L.load()
    cases = [(300, 4, 16, 1, L.SB_GROUP_POSITIVE_ONLY), (2048, 8, 128, 2, 0)]
    for n_rows, slots, groups, seed, flags in cases:
        idx, w = make_entries(n_rows, slots, groups, seed, cuda_device)
        ws = torch.zeros(lib.sb_group_workspace_bytes(n_rows, slots, groups), dtype=torch.uint8, device=cuda_device)
        want = outputs(n_rows, slots, groups, cuda_device)
        got = outputs(n_rows, slots, groups, cuda_device)
        call("sb_group", idx, w, n_rows, slots, groups, flags, want, ws)
        call("sb_group_noalloc", idx, w, n_rows, slots, groups, flags, got)
        torch.cuda.synchronize()
        used = int(want["offsets"][-1].item())
        assert torch.equal(got["offsets"], want["offsets"])
        assert torch.equal(got["inv"], want["inv"])
        for k in ("perm_row", "perm_slot", "perm_w"):
            assert torch.equal(got[k][:used], want[k][:used]), k


def test_noalloc_grouping_rejects_sizes_beyond_its_scratch(cuda_device):
    lib = L.load()
    n_rows, slots = MAX_ENTRIES // 4 + 1, 4
    idx = torch.zeros(n_rows, slots, dtype=torch.int32, device=cuda_device)
    w = torch.ones(n_rows, slots, device=cuda_device)
    out = outputs(n_rows, slots, 8, cuda_device)
    rc = lib.sb_group_noalloc(idx.data_ptr(), w.data_ptr(), n_rows, slots, 8, 0, out["offsets"].data_ptr(),
                              out["perm_row"].data_ptr(), out["perm_slot"].data_ptr(), out["perm_w"].data_ptr(),
                              out["inv"].data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == L.SB_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert int(out["offsets"][0].item()) == -7  # nothing was launched
