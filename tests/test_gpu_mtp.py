"""The MTP draft module on the GPU against the reference's golden drafts: from each
sequence's verify row that produced the next token, three batched draft steps give the
reference's drafts, and the last step's hidden state is within 1e-2 of the reference's."""
import numpy as np
import pytest
import torch

from oracle import model as om
from pilm_b200 import bindings as abi
from pilm_b200 import ckernel as ck
from pilm_b200.mtp import MTPDrafter, MTPWeights
from pilm_b200.qwen3 import Qwen3Shape, Qwen3Weights
from tests import _golden as G
from tests._gpu import REL_TOL, bf16_from_bits, bits_of, dev, f32_of_bits, rel_err

pytestmark = pytest.mark.gpu
VARIANTS = ["qwen3_w4g128", "qwen35_w4g128", "qwen3_w4g128_gqa4"]


@pytest.fixture(scope="module", autouse=True)
def _init():
    abi.init()
    yield


def shape_of(cfg: om.Qwen3Config) -> Qwen3Shape:
    return Qwen3Shape(hidden=cfg.hidden, layers=cfg.layers, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
                      head_dim=cfg.head_dim, intermediate=cfg.intermediate, vocab=cfg.vocab, eps=cfg.eps,
                      rope_theta=cfg.rope_theta, partial_rotary=cfg.partial_rotary, gated=cfg.gated,
                      gemma_norm=cfg.gemma_norm, block_size=cfg.block_size)


@pytest.mark.parametrize("linears", ["w4a16", "bf16"])
@pytest.mark.parametrize("variant", VARIANTS)
def test_drafts_match_reference(variant, linears):
    """Both draft-module options: the PILM_MTP_QUANTIZE=w4a16 linears and the reference's
    default bf16 linears, against the reference drafts of that option."""
    z = G.load(f"model_{variant}.npz")
    cfg, seed = G.model_config(z)
    shape = shape_of(cfg)
    w = Qwen3Weights.from_checkpoint(shape, om.make_checkpoint(cfg, seed), dev())
    mw = MTPWeights.from_checkpoint(shape, om.make_mtp_checkpoint(cfg, seed), dev(), linears=linears)
    sfx = "_bf16" if linears == "bf16" else ""
    drafter = MTPDrafter(mw, w, max_seqs=8, device=dev())
    B = G.num_seqs(z)
    rows, cu, acc, nxt = [], [0], [], []
    for b in range(B):
        h = z[f"b{b}.hidden"]
        rows.append(h)
        cu.append(cu[-1] + h.shape[0])
        a, t = G.ilist(z[f"b{b}.accept"])
        acc.append(a)
        nxt.append(t)
    hidden = bf16_from_bits(np.concatenate(rows))
    i32 = dict(dtype=torch.int32, device=dev())
    out = torch.full((3, B), -1, **i32)
    last = drafter.draft(hidden, torch.tensor(cu, **i32), torch.tensor(acc, **i32), torch.tensor(nxt, **i32), 3, out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(B):
        assert got[:, b].tolist() == G.ilist(z[f"b{b}.mtp_drafts{sfx}"]), f"sequence {b}"
        ref = f32_of_bits(z[f"b{b}.mtp_last_hidden{sfx}"])[0]
        assert rel_err(f32_of_bits(bits_of(last[b])), ref) <= REL_TOL


@pytest.mark.parametrize("M", [1, 3, 8, 9, 16, 24, 32, 40, 64, 70])
def test_bf16_linear_vs_fp32_reference(M):
    """ekernel_linear_bf16 against torch's fp32 product of the same bf16 tensors, rounded
    once: every GEMV tile (M <= 8, 16, 32, 64), slabs above 64 rows, split-K and a ragged N."""
    g = torch.Generator().manual_seed(M)
    for (N, K) in [(300, 512), (1000, 4096)]:
        x = torch.randn((M, K), generator=g).to(torch.bfloat16)
        w = (torch.randn((N, K), generator=g) * 0.02).to(torch.bfloat16)
        ref = (x.float() @ w.float().t()).to(torch.bfloat16)
        got = ck.linear_bf16(x.to(dev()), w.to(dev())).cpu()
        assert rel_err(got.float().numpy(), ref.float().numpy()) <= REL_TOL
        assert (got == ref).float().mean().item() >= 0.99


def test_fc_input_and_self_attention_kernels():
    """The two draft-only kernels against their definitions: gathered-row norms with torch-
    module rounding (plain and Gemma) and single-key attention (plain and gated)."""
    g = torch.Generator().manual_seed(3)
    H, V, B = 512, 300, 5
    hidden = (torch.randn((9, H), generator=g) * 3).to(torch.bfloat16)
    embed = (torch.randn((V, H), generator=g) * 0.05).to(torch.bfloat16)
    we = (torch.randn(H, generator=g) * 0.1 + 1).to(torch.bfloat16)
    wh = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    base, off, tok = [0, 2, 4, 6, 8], [1, 0, 1, 1, 0], [5, 299, 0, 17, 128]
    d = dev()
    i32 = dict(dtype=torch.int32, device=d)
    for gemma in (False, True):
        got = ck.mtp_fc_input_bf16(hidden.to(d), torch.tensor(base, **i32), torch.tensor(off, **i32), embed.to(d),
                                   torch.tensor(tok, **i32), we.to(d), wh.to(d), 1e-6, gemma).cpu()
        src = hidden[[b + o for b, o in zip(base, off)]]
        ref = torch.cat([om.rms_norm(embed[tok], we, 1e-6, gemma), om.rms_norm(src, wh, 1e-6, gemma)], dim=-1)
        assert rel_err(got.float().numpy(), ref.float().numpy()) <= REL_TOL
    nh, nkv, hd, R = 8, 2, 128, 3
    v = torch.randn((R, nkv * hd), generator=g).to(torch.bfloat16)
    gate = torch.randn((R, nh * hd), generator=g).to(torch.bfloat16)
    expand = v.view(R, nkv, 1, hd).expand(R, nkv, nh // nkv, hd).reshape(R, nh * hd)
    got = ck.self_attention_bf16(v.to(d), None, nh, nkv, hd).cpu()
    assert torch.equal(got, expand)
    got = ck.self_attention_bf16(v.to(d), gate.to(d), nh, nkv, hd).cpu()
    assert rel_err(got.float().numpy(), (expand * torch.sigmoid(gate)).float().numpy()) <= REL_TOL
