"""The allocation-free paged-attention entry point.

ekernel_paged_attention_verify_noalloc is for callers that cannot let a kernel
library allocate GPU memory: an engine whose allocator owns the whole device, a
serving loop that must never hit cudaMalloc's implicit synchronisation, or a host
written in another language that only hands over buffers it already owns.  It keeps
its split-KV partials in a fixed 8 MiB array inside the library and records a failed
page wait in a fixed device word there too.

The tests call it through the C ABI:
  * twice in a row with different inputs (the array keeps the previous call's
    contents), each result checked against ekernel_paged_attention_verify and against
    the oracle's attention, within the tolerance of the other GPU parity tests;
  * in a fresh process as the library's very first call, checking that the library
    made no device allocation of its own (its allocation counter stays at zero);
  * with a request whose partials would not fit in the array, which it refuses.
This file is collected last on purpose, and builds all of its own inputs, so it also
runs alone.
"""
import ctypes
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import model as om
from pilm_b200 import bindings as abi

ROOT = Path(__file__).resolve().parents[1]
REL_TOL = 1e-2  # same norm-wise tolerance as the other GPU parity tests (tests/_gpu.py)
SCRATCH_BYTES = 8 << 20
RECORD_BYTES = (128 + 2) * 4  # one split record: O[128] + (m, l), fp32


def _desc(B, T, max_q, nh, nkv, num_blocks, max_pages, max_ctx):
    return abi.PagedAttnDesc(B, T, max_q, nh, nkv, 128, 16, num_blocks, max_pages, max_ctx, (nh + 2 * nkv) * 128,
                             max_ctx + 1, 128, 1e-6, 0, 0)


def _case(seed, dev, nh=8, nkv=2, ctxs=(4100, 2051), qlens=(3, 3)):
    """Sequences whose contexts span many pages, so the call splits the KV range and
    really uses the scratch array.  Host copies are kept for the oracle."""
    g = torch.Generator().manual_seed(seed)
    hd, bs = 128, 16
    pages = [(c + bs - 1) // bs for c in ctxs]
    nb = sum(pages) + 4
    perm = torch.randperm(nb - 1, generator=g)[: sum(pages)] + 1
    tables, off = [], 0
    for p in pages:
        tables.append([int(x) for x in perm[off:off + p]])
        off += p
    maxp = max(pages)
    T = sum(qlens)
    cu = [0]
    for n in qlens:
        cu.append(cu[-1] + n)
    host = {
        "q": torch.randn((T, nh * hd), generator=g).to(torch.bfloat16),
        "k": torch.randn((nb, bs, nkv, hd), generator=g).to(torch.bfloat16),
        "v": torch.randn((nb, bs, nkv, hd), generator=g).to(torch.bfloat16),
        "tables": tables, "ctxs": list(ctxs), "cu": cu, "nh": nh, "nkv": nkv,
    }
    t = {
        "q": host["q"].to(dev), "k": host["k"].to(dev), "v": host["v"].to(dev),
        "bt": torch.tensor([x + [0] * (maxp - len(x)) for x in tables], dtype=torch.int32, device=dev),
        "cu": torch.tensor(cu, dtype=torch.int32, device=dev),
        "ctx": torch.tensor(list(ctxs), dtype=torch.int32, device=dev),
    }
    return _desc(len(ctxs), T, max(qlens), nh, nkv, nb, maxp, max(ctxs)), t, host


def _run(fn, desc, t):
    out = torch.empty_like(t["q"])
    rc = fn(ctypes.byref(desc), t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(), t["bt"].data_ptr(),
            t["cu"].data_ptr(), t["ctx"].data_ptr(), None, out.data_ptr())
    assert rc == 0, abi.last_error()
    return out


def _oracle(host):
    cfg = om.Qwen3Config(n_heads=host["nh"], n_kv_heads=host["nkv"])
    q = host["q"].view(-1, host["nh"], 128)
    cu = host["cu"]
    return torch.cat([om.attend(cfg, q[cu[b]:cu[b + 1]], None, host["k"], host["v"], host["tables"][b],
                                host["ctxs"][b], True) for b in range(len(host["ctxs"]))])


def _rel(got, ref):
    g, r = got.float().cpu().numpy(), ref.float().cpu().numpy()
    return float(np.abs(g - r).max() / max(np.abs(r).max(), 1e-30))


@pytest.mark.gpu
def test_noalloc_attention_matches_allocating_entry_two_calls():
    abi.init()
    dev = torch.device("cuda:0")
    abi.set_stream(torch.cuda.current_stream().cuda_stream)
    lib = abi.lib()
    for seed in (11, 12):  # two calls in a row, different inputs
        desc, t, host = _case(seed, dev)
        ref = _run(lib.ekernel_paged_attention_verify, desc, t)
        got = _run(lib.ekernel_paged_attention_verify_noalloc, desc, t)
        torch.cuda.synchronize()
        err = _rel(got, ref)
        assert err <= REL_TOL, f"call with seed {seed}: relative error {err} against the allocating entry point"
        err = _rel(got, _oracle(host))
        assert err <= REL_TOL, f"call with seed {seed}: relative error {err} against the oracle"


_FIRST_CALL = r"""
import ctypes, sys, torch
sys.path.insert(0, sys.argv[1])
from tests.test_zz_no_alloc import _case, _run, _rel, _oracle
from pilm_b200 import bindings as abi
abi.init()
dev = torch.device("cuda:0")
abi.set_stream(torch.cuda.current_stream().cuda_stream)
lib = abi.lib()
assert abi.alloc_count() == 0, abi.alloc_count()
for seed in (21, 22):
    desc, t, host = _case(seed, dev)
    torch.cuda.synchronize()
    got = _run(lib.ekernel_paged_attention_verify_noalloc, desc, t)
    torch.cuda.synchronize()
    n = abi.alloc_count()
    assert n == 0, f"the library allocated {n} time(s) during an allocation-free call"
    err = _rel(got, _oracle(host))
    assert err <= 1e-2, err
print("NOALLOC_FIRST_OK")
"""


@pytest.mark.gpu
def test_noalloc_first_call_in_a_fresh_process_allocates_nothing():
    """As the first library call of a process (no allocating entry point has run), two
    allocation-free calls leave the library's allocation counter at zero."""
    r = subprocess.run([sys.executable, "-c", _FIRST_CALL, str(ROOT)], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, PYTHONPATH=str(ROOT)))
    assert r.returncode == 0 and "NOALLOC_FIRST_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def _planned_records(desc, sms):
    """The split plan of the per-head attention kernel (attention.cu plan_splits): split
    records = splits x total_q x n_heads when the KV range is split."""
    kwarps = 4
    gsz = desc.n_heads // desc.n_kv_heads
    rows = (desc.max_q_len or 1) * gsz
    mt = 2 if rows > 16 else 1
    row_chunks = (rows + 16 * mt - 1) // (16 * mt)
    max_pages = (desc.max_context + 15) // 16
    base = desc.num_seqs * desc.n_kv_heads * row_chunks
    splits = (4 * sms + base - 1) // base
    splits = max(1, min(splits, max(1, max_pages // (2 * kwarps))))
    pps = max(1, (max_pages + splits - 1) // splits)
    splits = max(1, (max_pages + pps - 1) // pps)
    return splits * desc.total_q * desc.n_heads if splits > 1 else 0


@pytest.mark.gpu
def test_noalloc_rejects_requests_beyond_its_fixed_scratch():
    """One sequence of 64 query rows, 32 query / 8 KV heads, 32768 keys: on a 148-SM
    B200 the plan is 10 splits, i.e. 10 x 64 x 32 records x 520 B = 10.6 MB > 8 MiB, so
    the call is refused before any launch.  The buffers are real and sized for the
    request, so on a GPU whose plan fits the call would simply run."""
    abi.init()
    dev = torch.device("cuda:0")
    abi.set_stream(torch.cuda.current_stream().cuda_stream)
    nh, nkv, ctx, ql = 32, 8, 32768, 64
    pages = ctx // 16
    nb = pages + 1
    desc = _desc(1, ql, ql, nh, nkv, nb, pages, ctx)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    need = _planned_records(desc, sms) * RECORD_BYTES
    t = {
        "q": torch.zeros((ql, nh * 128), dtype=torch.bfloat16, device=dev),
        "k": torch.zeros((nb, 16, nkv, 128), dtype=torch.bfloat16, device=dev),
        "v": torch.zeros((nb, 16, nkv, 128), dtype=torch.bfloat16, device=dev),
        "bt": torch.arange(1, pages + 1, dtype=torch.int32, device=dev).view(1, pages),
        "cu": torch.tensor([0, ql], dtype=torch.int32, device=dev),
        "ctx": torch.tensor([ctx], dtype=torch.int32, device=dev),
    }
    out = torch.empty_like(t["q"])
    lib = abi.lib()
    rc = lib.ekernel_paged_attention_verify_noalloc(ctypes.byref(desc), t["q"].data_ptr(), t["k"].data_ptr(),
                                                    t["v"].data_ptr(), t["bt"].data_ptr(), t["cu"].data_ptr(),
                                                    t["ctx"].data_ptr(), None, out.data_ptr())
    torch.cuda.synchronize()
    if need > SCRATCH_BYTES:
        assert rc == -1
        msg = abi.last_error()
        assert f"needs {need} bytes" in msg and "at most 8388608 bytes" in msg, msg
    else:
        assert rc == 0, abi.last_error()
