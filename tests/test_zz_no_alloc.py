"""The allocation-free paged-attention entry point.

ekernel_paged_attention_verify_noalloc serves callers that cannot let a kernel
library allocate GPU memory (an engine whose allocator owns the device, a serving
loop that must not hit cudaMalloc's implicit synchronisation, a host language that
only passes in buffers it owns).  It keeps its split-KV partials in a fixed 8 MiB
array inside the library.  The GPU test calls it twice in a row through the C ABI,
with different inputs each time (the array keeps the previous call's contents), and
compares each result with ekernel_paged_attention_verify.  This file is collected
last on purpose; it builds all of its own inputs so it also runs alone.
"""
import ctypes

import numpy as np
import pytest
import torch

from pilm_b200 import bindings as abi

REL_TOL = 1e-2  # same norm-wise tolerance as the other GPU parity tests (tests/_gpu.py)


def _desc(B, T, max_q, nh, nkv, num_blocks, max_pages, max_ctx):
    return abi.PagedAttnDesc(B, T, max_q, nh, nkv, 128, 16, num_blocks, max_pages, max_ctx, (nh + 2 * nkv) * 128,
                             max_ctx + 1, 128, 1e-6, 0, 0)


def _case(seed, dev):
    """Two sequences whose contexts span many pages, so the call splits the KV range
    and really uses the scratch array."""
    g = torch.Generator().manual_seed(seed)
    nh, nkv, hd, bs = 8, 2, 128, 16
    ctxs, qlens = [4100, 2051], [3, 3]
    pages = [(c + bs - 1) // bs for c in ctxs]
    nb = sum(pages) + 4
    perm = torch.randperm(nb - 1, generator=g)[: sum(pages)] + 1
    tables, off = [], 0
    for p in pages:
        tables.append([int(x) for x in perm[off:off + p]])
        off += p
    maxp = max(pages)
    T = sum(qlens)
    t = {
        "q": torch.randn((T, nh * hd), generator=g).to(torch.bfloat16).to(dev),
        "k": torch.randn((nb, bs, nkv, hd), generator=g).to(torch.bfloat16).to(dev),
        "v": torch.randn((nb, bs, nkv, hd), generator=g).to(torch.bfloat16).to(dev),
        "bt": torch.tensor([x + [0] * (maxp - len(x)) for x in tables], dtype=torch.int32, device=dev),
        "cu": torch.tensor([0, qlens[0], T], dtype=torch.int32, device=dev),
        "ctx": torch.tensor(ctxs, dtype=torch.int32, device=dev),
    }
    return _desc(2, T, max(qlens), nh, nkv, nb, maxp, max(ctxs)), t


def _run(fn, desc, t):
    out = torch.empty_like(t["q"])
    rc = fn(ctypes.byref(desc), t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(), t["bt"].data_ptr(),
            t["cu"].data_ptr(), t["ctx"].data_ptr(), None, out.data_ptr())
    assert rc == 0, abi.last_error()
    return out


@pytest.mark.gpu
def test_noalloc_attention_matches_allocating_entry_two_calls():
    abi.init()
    dev = torch.device("cuda:0")
    abi.set_stream(torch.cuda.current_stream().cuda_stream)
    lib = abi.lib()
    for seed in (11, 12):  # two calls in a row, different inputs
        desc, t = _case(seed, dev)
        ref = _run(lib.ekernel_paged_attention_verify, desc, t)
        got = _run(lib.ekernel_paged_attention_verify_noalloc, desc, t)
        torch.cuda.synchronize()
        r, o = ref.float().cpu().numpy(), got.float().cpu().numpy()
        err = float(np.abs(o - r).max() / max(np.abs(r).max(), 1e-30))
        assert err <= REL_TOL, f"call with seed {seed}: relative error {err}"


def test_noalloc_rejects_requests_beyond_its_fixed_scratch():
    """Needs 32 splits x 64 rows x 8 heads x 520 B > 8 MiB: refused before any launch
    (argument checking only; the pointers are never used)."""
    lib = abi.lib()
    desc = _desc(4, 64, 16, 8, 2, 2000, 300, 4800)
    dummy = ctypes.c_void_p(16)
    rc = lib.ekernel_paged_attention_verify_noalloc(ctypes.byref(desc), dummy, dummy, dummy, dummy, dummy, dummy,
                                                    None, dummy)
    assert rc == -1
    assert "at most 8388608 bytes" in abi.last_error()
