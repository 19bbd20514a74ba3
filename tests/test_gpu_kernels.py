"""GPU parity of the quantized linears, norms and SwiGLU against the reference's
golden outputs and the pinned oracle, through the C ABI (pilm_b200.bindings)."""
import numpy as np
import pytest
import torch

from oracle import kernels as ok
from pilm_b200 import bindings as abi
from pilm_b200 import ckernel as ck
from tests import _golden as G
from tests._gpu import REL_TOL, assert_bf16_close, bf16_from_bits, bits_of, dev, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    abi.init()
    yield


@pytest.fixture(scope="module")
def kz():
    return G.load("kernels.npz")


def _shapes(kz):
    return sorted({k.split(".")[0] for k in kz.files if k.startswith("s") and k.endswith(".shape")})


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev())
    return t if dtype is None else t.to(dtype)


def test_linears_vs_reference_golden(kz):
    for s in _shapes(kz):
        x = bf16_from_bits(kz[f"{s}.x"])
        for grp, fn in ((128, ck.linear_w4a16g128_bf16), (32, ck.linear_w4a16g32_bf16)):
            y = fn(x, _t(kz[f"{s}.w4g{grp}.qw"]), _t(kz[f"{s}.w4g{grp}.s"]))
            assert_bf16_close(bits_of(y), kz[f"{s}.w4g{grp}.y"], ulp_frac=0.99)
        y = ck.linear_w4a16_bf16(x, _t(kz[f"{s}.w4row.qw"]), _t(kz[f"{s}.w4row.s"]))
        assert_bf16_close(bits_of(y), kz[f"{s}.w4row.y"], ulp_frac=0.99)
        y = ck.linear_w8a16_bf16(x, _t(kz[f"{s}.w8.qw"]), _t(kz[f"{s}.w8.s"]))
        assert_bf16_close(bits_of(y), kz[f"{s}.w8a16.y"], ulp_frac=0.99)
        y = ck.linear_w8a32(_t(kz[f"{s}.xf"]), _t(kz[f"{s}.w8.qw"]), _t(kz[f"{s}.w8.s"]))
        assert rel_err(y.cpu().numpy(), kz[f"{s}.w8a32.y"]) <= 1e-5


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 12, 16, 24, 32, 48, 63, 64, 96, 100, 128, 130, 256])
@pytest.mark.parametrize("NK", [(256, 512), (384, 1024), (200, 4096), (136, 1152), (100, 2048)])
def test_w4g128_vs_oracle_all_regimes(M, NK):
    """Both GEMV tile configurations (M <= 8, 16) and the tensor-core path above 16 rows
    (N = 32, 48, 64, ... activation rows per MMA), including split-K (K=4096), ragged N,
    an N that is not a multiple of 8 (no split-K
    combine pass), and a group count that is not a multiple of 4 (K=1152: the tensor-core
    path loads group scales directly instead of by TMA)."""
    N, K = NK
    rng = np.random.default_rng(M * 7 + N)
    x = ok.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    qw, s = ok.quantize_i4_grouped(w, 128)
    ref = ok.linear_w4a16g_bf16(x, qw, s, 128)
    y = ck.linear_w4a16g128_bf16(bf16_from_bits(x), _t(qw), _t(s))
    assert_bf16_close(bits_of(y), ref, ulp_frac=0.99)
    qr, sr = ok.quantize_i4_per_row(w)
    ref = ok.linear_w4a16_bf16(x, qr, sr)
    y = ck.linear_w4a16_bf16(bf16_from_bits(x), _t(qr), _t(sr))
    assert_bf16_close(bits_of(y), ref, ulp_frac=0.99)


@pytest.mark.parametrize("M", [64, 96, 128, 200])
def test_large_m_qwen3_8b_shapes(M):
    """The M >= 64 tensor-core path on the Qwen3-8B projection shapes that fit a test:
    fused QKV (4096 -> 6144) and down (12288 -> 4096), one activation tile (M <= 128)
    and two (M = 200), with and without split-K.  Each shape runs three times in a row:
    the pipeline's warps race one another, and a result that depends on their timing
    differs between calls."""
    rng = np.random.default_rng(M)
    for (N, K) in [(6144, 4096), (4096, 12288)]:
        x = ok.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        qw, s = ok.quantize_i4_grouped(w, 128)
        ref = ok.linear_w4a16g_bf16(x, qw, s, 128)
        xd, qd, sd = bf16_from_bits(x), _t(qw), _t(s)
        for _ in range(3):
            y = ck.linear_w4a16g128_bf16(xd, qd, sd)
            assert_bf16_close(bits_of(y), ref, ulp_frac=0.99)


@pytest.mark.parametrize("inter", [512, 12288, 100])
def test_silu_mul_vector_path_matches_scalar(inter):
    """silu(gate) * up with torch-module rounding: the 8-wide kernel (aligned rows, inter %
    8 == 0) gives the scalar kernel's bits (an output offset by one element takes the
    scalar kernel), and both stay within 1e-2 of the fp32 formula."""
    g = torch.Generator().manual_seed(inter)
    gu = (torch.randn((7, 2 * inter), generator=g) * 3).to(torch.bfloat16).to(dev())
    fast = ck.silu_mul_bf16(gu, inter)
    buf = torch.empty(7 * inter + 1, dtype=torch.bfloat16, device=dev())
    slow = ck.silu_mul_bf16(gu, inter, out=buf[1:].view(7, inter))
    assert torch.equal(fast.cpu(), slow.cpu())
    gf, uf = gu[:, :inter].float().cpu(), gu[:, inter:].float().cpu()
    ref = (gf / (1 + torch.exp(-gf))) * uf
    assert rel_err(fast.float().cpu().numpy(), ref.numpy()) <= REL_TOL


def test_kpairs_repack_and_linears():
    """The k-pair repack is the oracle's nibble permutation bit for bit (in place too), and
    both W4 linears on repacked weights match the oracle on the reference packing: the
    GEMV tiles (M <= 8, 16) and the tensor-core path, with and without split-K."""
    rng = np.random.default_rng(11)
    for (N, K) in [(384, 1024), (200, 4096)]:
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        qw, s = ok.quantize_i4_grouped(w, 128)
        qr, sr = ok.quantize_i4_per_row(w)
        want = ok.repack_w4_kpairs(qw)
        qd = _t(qw)
        got = ck.repack_w4_kpairs(qd)
        assert np.array_equal(got.cpu().numpy(), want)
        inplace = qd.clone()
        ck.repack_w4_kpairs(inplace, out=inplace)
        assert np.array_equal(inplace.cpu().numpy(), want)
        qrd = ck.repack_w4_kpairs(_t(qr))
        for M in (1, 5, 16, 24, 96, 200):
            x = ok.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
            xd = bf16_from_bits(x)
            y = ck.linear_w4a16g128_bf16(xd, got, _t(s), kpairs=True)
            assert_bf16_close(bits_of(y), ok.linear_w4a16g_bf16(x, qw, s, 128), ulp_frac=0.99)
            y = ck.linear_w4a16_bf16(xd, qrd, _t(sr), kpairs=True)
            assert_bf16_close(bits_of(y), ok.linear_w4a16_bf16(x, qr, sr), ulp_frac=0.99)


@pytest.mark.parametrize("M", [24, 96])
@pytest.mark.parametrize("K", [512, 1152])
def test_stream_k_schedule_vs_oracle(M, K):
    """At least one 128-row tile per SM selects the stream-K schedule: every CTA runs an equal
    range of (tile, group) units, so range boundaries cut tiles and the cut pieces are
    summed in the kernel by the last CTA to arrive.  149 tiles with a ragged last one
    (N = 19000) over 4 or 9 groups cut nearly every tile; K = 1152 also takes the group
    scales without TMA.  Both weight layouts, twice in a row (the per-tile arrival counters
    reset themselves)."""
    N = 19000
    rng = np.random.default_rng(M + K)
    x = ok.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    qw, s = ok.quantize_i4_grouped(w, 128)
    ref = ok.linear_w4a16g_bf16(x, qw, s, 128)
    xd, qd, sd = bf16_from_bits(x), _t(qw), _t(s)
    qk = ck.repack_w4_kpairs(qd)
    for _ in range(2):
        assert_bf16_close(bits_of(ck.linear_w4a16g128_bf16(xd, qd, sd)), ref, ulp_frac=0.99)
        assert_bf16_close(bits_of(ck.linear_w4a16g128_bf16(xd, qk, sd, kpairs=True)), ref, ulp_frac=0.99)


def test_kpairs_refuses_ragged_k():
    rng = np.random.default_rng(12)
    w = (rng.standard_normal((16, 200)) * 0.02).astype(np.float32)
    qw, s = ok.quantize_i4_grouped(w, 128)
    x = bf16_from_bits(ok.f32_to_bf16(rng.standard_normal((3, 200)).astype(np.float32)))
    with pytest.raises(RuntimeError, match="kpairs"):
        ck.linear_w4a16g128_bf16(x, ck.repack_w4_kpairs(_t(qw)), _t(s), kpairs=True)


def test_ragged_k_falls_back_and_matches():
    rng = np.random.default_rng(3)
    for (M, N, K) in [(3, 17, 130), (1, 5, 77), (6, 33, 200)]:
        x = ok.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        qw, s = ok.quantize_i4_grouped(w, 128)
        y = ck.linear_w4a16g128_bf16(bf16_from_bits(x), _t(qw), _t(s))
        assert_bf16_close(bits_of(y), ok.linear_w4a16g_bf16(x, qw, s, 128), ulp_frac=0.99)


def test_rmsnorm_and_swiglu_vs_golden(kz):
    for s in _shapes(kz):
        for add_one in (0, 1):
            y = ck.rmsnorm_bf16(bf16_from_bits(kz[f"{s}.x"]), bf16_from_bits(kz[f"{s}.norm.w"]), 1e-6, bool(add_one))
            assert_bf16_close(bits_of(y), kz[f"{s}.norm{add_one}.y"], ulp_frac=0.99)
    y = ck.swiglu_bf16(bf16_from_bits(kz["swiglu.g"]), bf16_from_bits(kz["swiglu.u"]))
    assert_bf16_close(bits_of(y), kz["swiglu.y"], ulp_frac=0.99)
    H, I, K = [int(v) for v in kz["mlp.dims"]]
    y = ck.swiglu_w4a16_bf16(bf16_from_bits(kz["mlp.x"]), _t(kz["mlp.gu_qw"]), _t(kz["mlp.gu_s"]),
                             _t(kz["mlp.d_qw"]), _t(kz["mlp.d_s"]), I)
    assert_bf16_close(bits_of(y), kz["mlp.y"], ulp_frac=0.98)


def test_fused_swiglu_any_m_vs_oracle():
    rng = np.random.default_rng(5)
    H, I, K, M = 256, 384, 512, 5
    x = ok.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    gq, gs = ok.quantize_i4_per_row((rng.standard_normal((2 * I, K)) * 0.02).astype(np.float32))
    dq, ds = ok.quantize_i4_per_row((rng.standard_normal((H, I)) * 0.02).astype(np.float32))
    ref = np.concatenate([ok.swiglu_w4a16_bf16(x[m], gq, gs, dq, ds, I) for m in range(M)])
    y = ck.swiglu_w4a16_bf16(bf16_from_bits(x), _t(gq), _t(gs), _t(dq), _t(ds), I)
    assert_bf16_close(bits_of(y), ref, ulp_frac=0.98)


def test_gemm_known_answer_and_argmax():
    a = torch.tensor([[1, 2], [3, 4]], dtype=torch.float32, device=dev())
    b = torch.tensor([[5, 6], [7, 8]], dtype=torch.float32, device=dev())
    assert ck.gemm_f32(a, b).cpu().tolist() == [[19, 22], [43, 50]]
    rng = np.random.default_rng(9)
    x = ok.f32_to_bf16(rng.standard_normal((1, 256)).astype(np.float32))
    q8, s8 = ok.quantize_i8_per_row((rng.standard_normal((1000, 256)) * 0.02).astype(np.float32))
    idx_ref, _ = ok.linear_w8a16_bf16_argmax(x, q8, s8)
    assert ck.linear_w8a16_bf16_argmax(bf16_from_bits(x), _t(q8), _t(s8)) == idx_ref


def test_sync_mode_reports_ok_and_errors_are_strings():
    assert abi.lib().ekernel_synchronize() == 0
