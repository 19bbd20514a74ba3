"""CPU tests: pin the oracle (oracle/) against the reference's golden fixtures
and, where the reference library was built here, against it directly."""
import hashlib

import numpy as np
import pytest
import torch

from oracle import kernels as ok
from oracle import model as om
from oracle import reflib
from tests import _golden as G


@pytest.fixture(scope="module")
def kz():
    return G.load("kernels.npz")


def _shapes(kz):
    return sorted({k.split(".")[0] for k in kz.files if k.startswith("s") and k.endswith(".shape")})


def test_quantizers_match_reference(kz):
    for s in _shapes(kz):
        w = kz[f"{s}.w"]
        for grp in (32, 128):
            qw, sc = ok.quantize_i4_grouped(w, grp)
            assert np.array_equal(qw, kz[f"{s}.w4g{grp}.qw"]) and np.array_equal(sc, kz[f"{s}.w4g{grp}.s"])
        qw, sc = ok.quantize_i4_per_row(w)
        assert np.array_equal(qw, kz[f"{s}.w4row.qw"]) and np.array_equal(sc, kz[f"{s}.w4row.s"])
        q8, s8 = ok.quantize_i8_per_row(w)
        assert np.array_equal(q8, kz[f"{s}.w8.qw"]) and np.array_equal(s8, kz[f"{s}.w8.s"])


def test_linear_kernels_bit_exact(kz):
    for s in _shapes(kz):
        x, xf = kz[f"{s}.x"], kz[f"{s}.xf"]
        for grp in (32, 128):
            y = ok.linear_w4a16g_bf16(x, kz[f"{s}.w4g{grp}.qw"], kz[f"{s}.w4g{grp}.s"], grp)
            assert np.array_equal(y, kz[f"{s}.w4g{grp}.y"]), (s, grp)
        assert np.array_equal(ok.linear_w4a16_bf16(x, kz[f"{s}.w4row.qw"], kz[f"{s}.w4row.s"]), kz[f"{s}.w4row.y"])
        assert np.array_equal(ok.linear_w8a16_bf16(x, kz[f"{s}.w8.qw"], kz[f"{s}.w8.s"]), kz[f"{s}.w8a16.y"])
        assert np.array_equal(ok.linear_w8a32(xf, kz[f"{s}.w8.qw"], kz[f"{s}.w8.s"]).view(np.uint32),
                              kz[f"{s}.w8a32.y"].view(np.uint32))


def test_norm_and_swiglu_bit_exact(kz):
    for s in _shapes(kz):
        for add_one in (0, 1):
            y = ok.rmsnorm_bf16(kz[f"{s}.x"], kz[f"{s}.norm.w"], 1e-6, add_one)
            assert np.array_equal(y, kz[f"{s}.norm{add_one}.y"])
    assert np.array_equal(ok.swiglu_bf16(kz["swiglu.g"], kz["swiglu.u"]), kz["swiglu.y"])
    H, I, K = [int(v) for v in kz["mlp.dims"]]
    y = ok.swiglu_w4a16_bf16(kz["mlp.x"], kz["mlp.gu_qw"], kz["mlp.gu_s"], kz["mlp.d_qw"], kz["mlp.d_s"], I)
    assert np.array_equal(y, kz["mlp.y"])


def test_gemm_known_answer():
    """src/ecpu/test/base_test.c:38-41: [[1,2],[3,4]] @ [[5,6],[7,8]] == [[19,22],[43,50]]."""
    c = ok.gemm_f32(np.array([[1, 2], [3, 4]], np.float32), np.array([[5, 6], [7, 8]], np.float32))
    assert c.tolist() == [[19, 22], [43, 50]]


@pytest.mark.skipif(not reflib.available(), reason="reference library not built here")
def test_oracle_vs_reference_library_random_shapes():
    rng = np.random.default_rng(11)
    for _ in range(25):
        M, N, K = int(rng.integers(1, 20)), int(rng.integers(1, 300)), int(rng.integers(1, 700))
        x = ok.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32) * np.float32(rng.uniform(0.1, 5)))
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        for grp in (32, 128):
            qw, s = ok.quantize_i4_grouped(w, grp)
            assert np.array_equal(ok.linear_w4a16g_bf16(x, qw, s, grp), reflib.linear(f"w4a16g{grp}_bf16", x, qw, s))
        q8, s8 = ok.quantize_i8_per_row(w)
        xf = rng.standard_normal((M, K)).astype(np.float32)
        assert np.array_equal(ok.linear_w8a32(xf, q8, s8).view(np.uint32), reflib.linear("w8a32", xf, q8, s8).view(np.uint32))


@pytest.mark.skipif(not reflib.available(), reason="reference library not built here")
def test_oracle_vs_reference_library_other_kernels_random_shapes():
    """The rest of the restated C kernels (the W8A16 LM-head argmax included) against the
    reference library, bit for bit, on random shapes: ragged K (AVX2 tails of 1-7 values), odd K (a half-filled last byte of
    packed int4), rows of any width for the norm, and scaled activations."""
    rng = np.random.default_rng(23)
    for _ in range(20):
        M, N, K = int(rng.integers(1, 12)), int(rng.integers(1, 200)), int(rng.integers(1, 600))
        x = ok.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32) * np.float32(rng.uniform(0.1, 5)))
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        qr, sr = ok.quantize_i4_per_row(w)
        assert np.array_equal(ok.linear_w4a16_bf16(x, qr, sr), reflib.linear("w4a16_bf16", x, qr, sr))
        q8, s8 = ok.quantize_i8_per_row(w)
        assert np.array_equal(ok.linear_w8a16_bf16(x, q8, s8), reflib.linear("w8a16_bf16", x, q8, s8))
        got, want = ok.linear_w8a16_bf16_argmax(x[:1], q8, s8), reflib.linear_w8a16_bf16_argmax(x[:1], q8, s8)
        assert got[0] == want[0] and np.float32(got[1]).view(np.uint32) == np.float32(want[1]).view(np.uint32)
        n = int(rng.integers(1, 700))
        xr = ok.f32_to_bf16(rng.standard_normal((M, n)).astype(np.float32) * np.float32(rng.uniform(0.01, 30)))
        wn = ok.f32_to_bf16((1 + 0.1 * rng.standard_normal(n)).astype(np.float32))
        for add_one in (False, True):
            assert np.array_equal(ok.rmsnorm_bf16(xr, wn, 1e-6, add_one), reflib.rmsnorm_bf16(xr, wn, 1e-6, add_one))
        g = ok.f32_to_bf16(rng.standard_normal(n).astype(np.float32) * 4)
        u = ok.f32_to_bf16(rng.standard_normal(n).astype(np.float32))
        assert np.array_equal(ok.swiglu_bf16(g, u), reflib.swiglu_bf16(g, u))
    for H, inter in ((64, 96), (40, 136), (128, 256)):
        x1 = ok.f32_to_bf16(rng.standard_normal((1, H)).astype(np.float32))
        gu, gus = ok.quantize_i4_grouped((rng.standard_normal((2 * inter, H)) * 0.02).astype(np.float32), 128)
        dq, ds = ok.quantize_i4_grouped((rng.standard_normal((H, inter)) * 0.02).astype(np.float32), 128)
        assert np.array_equal(ok.swiglu_w4a16_bf16(x1, gu, gus, dq, ds, inter),
                              reflib.swiglu_w4a16_bf16(x1, gu, gus, dq, ds, inter))


@pytest.mark.parametrize("variant", G.MODEL_VARIANTS)
def test_oracle_model_matches_reference_trace(variant):
    """Replays the reference's prefill chunk schedule, then the verify step: hidden,
    logits, accept counts and the weight checksum equal the reference's bit for bit."""
    z = G.load(f"model_{variant}.npz")
    cfg, seed = G.model_config(z)
    ck = om.make_checkpoint(cfg, seed)
    m = om.OracleModel(cfg, ck)
    h = hashlib.sha256()
    for key in sorted(m.q):
        h.update(m.q[key]["qweight"].tobytes())
        h.update(m.q[key]["scales"].tobytes())
    assert np.frombuffer(h.digest(), np.uint8).tolist() == z["qweights_sha256"].tolist()
    B = G.num_seqs(z)
    kvk, kvv = m.new_kv(32)
    prompts = [G.ilist(z[f"b{b}.prompt"]) for b in range(B)]
    tables = [G.ilist(z[f"b{b}.block_ids"]) for b in range(B)]
    m.replay_chunks(prompts, z["prefill_chunks"], kvk, kvv, tables)
    for li in range(cfg.layers):
        got = kvk[li].view(torch.int16).numpy().view(np.uint16) if cfg.dtype == "bfloat16" else kvk[li].numpy()
        assert np.array_equal(got, z[f"kv.k{li}"])
    for b in range(B):
        hid = m.forward(G.ilist(z[f"b{b}.verify_ids"]), G.ilist(z[f"b{b}.positions"]), kvk, kvv, tables[b], True)
        lg = m.logits(hid)
        assert np.array_equal(lg.numpy().view(np.uint32), z[f"b{b}.logits"].view(np.uint32))
        acc, nxt = om.greedy_accept(lg, G.ilist(z[f"b{b}.drafts"]))
        assert [acc, nxt] == G.ilist(z[f"b{b}.accept"])
        if f"b{b}.recompute_hidden_last" in z.files:
            # the reference re-runs the accepted prefix after a rejection; the last row
            # equals the verify row at the same position (recompute-free reject path)
            # (bit-identical in bf16; fp32 bmm depends on the row count: ~1e-7 relative)
            row = hid[acc:acc + 1]
            if cfg.dtype == "bfloat16":
                got = row.view(torch.int16).numpy().view(np.uint16)
                assert np.array_equal(got, z[f"b{b}.recompute_hidden_last"])
            else:
                np.testing.assert_allclose(row.numpy(), z[f"b{b}.recompute_hidden_last"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("variant", [v for v in G.MODEL_VARIANTS if "w4g128" in v])
def test_oracle_mtp_drafts_match_reference(variant):
    """The W4A16 MTP draft module: from each sequence's verify row that produced the next
    token (its normed hidden state and that token), three draft steps give the reference's
    drafts, and the last step's hidden state equals the reference's bit for bit."""
    z = G.load(f"model_{variant}.npz")
    cfg, seed = G.model_config(z)
    m = om.OracleModel(cfg, om.make_checkpoint(cfg, seed))
    mck = om.make_mtp_checkpoint(cfg, seed)
    mtp = om.OracleMTP(cfg, mck, m)
    h = hashlib.sha256()
    for key in sorted(mtp.q):
        h.update(mtp.q[key]["qweight"].tobytes())
        h.update(mtp.q[key]["scales"].tobytes())
    assert np.frombuffer(h.digest(), np.uint8).tolist() == z["mtp_qweights_sha256"].tolist()
    for b in range(G.num_seqs(z)):
        acc, nxt = G.ilist(z[f"b{b}.accept"])
        hid = om._from_bits(z[f"b{b}.hidden"])[acc]
        drafts, last = mtp.draft_tokens(hid, nxt, 3)
        assert drafts == G.ilist(z[f"b{b}.mtp_drafts"])
        assert np.array_equal(om._to_bits(last.reshape(1, -1)), z[f"b{b}.mtp_last_hidden"])


@pytest.mark.parametrize("variant", [v for v in G.MODEL_VARIANTS if "w4g128" in v])
def test_oracle_mtp_bf16_drafts_match_reference(variant):
    """The draft module with the reference's default bf16 linears: the same three draft
    steps give the reference's drafts and its last hidden state bit for bit."""
    z = G.load(f"model_{variant}.npz")
    cfg, seed = G.model_config(z)
    m = om.OracleModel(cfg, om.make_checkpoint(cfg, seed))
    mtp = om.OracleMTP(cfg, om.make_mtp_checkpoint(cfg, seed), m, linears="bf16")
    for b in range(G.num_seqs(z)):
        acc, nxt = G.ilist(z[f"b{b}.accept"])
        hid = om._from_bits(z[f"b{b}.hidden"])[acc]
        drafts, last = mtp.draft_tokens(hid, nxt, 3)
        assert drafts == G.ilist(z[f"b{b}.mtp_drafts_bf16"])
        assert np.array_equal(om._to_bits(last.reshape(1, -1)), z[f"b{b}.mtp_last_hidden_bf16"])


def test_draft_limit_matches_engine_rule():
    # engine.py:399-401
    assert om.draft_limit(21, 16, 64, 3) == 3
    assert om.draft_limit(30, 16, 64, 3) == 1
    assert om.draft_limit(31, 16, 64, 3) == 0
    assert om.draft_limit(32, 16, 2, 3) == 2
    assert om.draft_limit(5, 16, 0, 3) == 0


def test_rejection_sampling_restatement_properties():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(4, 50, generator=g) * 3
    p = om.nucleus_probs(logits[0], 0.8, 0.95)
    assert abs(float(p.sum()) - 1.0) < 1e-9
    # accept probability of a draft equals its nucleus probability
    d = int(torch.argmax(logits[0]))
    acc, _ = om.rejection_accept(logits, [d], [float(p[d]) - 1e-6], [0.5, 0.5], 0.8, 0.95)
    assert acc == 1
    acc, nxt = om.rejection_accept(logits, [d], [float(p[d]) + 1e-6], [0.5, 0.5], 0.8, 0.95)
    assert acc == 0 and nxt != d


def test_kpairs_repack_is_a_nibble_permutation():
    """The checker for the GPU library's k-pair layout only moves nibbles within 32-bit
    words: unpacking it and undoing the permutation gives the reference packing back."""
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((7, 256)) * 0.02).astype(np.float32)
    qw, _ = ok.quantize_i4_grouped(w, 128)
    kp = ok.repack_w4_kpairs(qw)
    nib = np.empty((7, 256), np.uint8)
    nib[:, 0::2] = kp & 15
    nib[:, 1::2] = kp >> 4
    words = nib.reshape(7, -1, 8)
    back = np.empty_like(words)
    back[:, :, list(ok.KPAIRS_ORDER)] = words
    back = back.reshape(7, -1)
    assert np.array_equal((back[:, 0::2] | (back[:, 1::2] << 4)).astype(np.uint8), qw)
    assert not np.array_equal(kp, qw)
