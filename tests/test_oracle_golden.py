"""The CPU oracle against golden vectors produced by the reference (tests/golden/make_golden.py)."""

import numpy as np
import pytest
import torch

from oracle import ngpt_oracle as O
from tests.helpers import CFG1, CFG3, CFG4, SMALL, fingerprint, row_rel_err, seeded_model, state_numpy


def test_rotary_tables_match_reference(golden):
    g = golden("ops_small.npz")
    cos, sin = O.rotary_frequencies(2048, 64, 10000.0, dtype=np.float32)
    np.testing.assert_allclose(cos, g["rope2048_cos"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(sin, g["rope2048_sin"], atol=2e-6, rtol=0)


@pytest.mark.parametrize("tag", ["even", "odd"])
def test_qkv_postprocess_matches_reference(golden, tag):
    g = golden("ops_small.npz")
    q, k, v = O.qkv_postprocess_from_carried(g[f"qkv_{tag}_in"], g[f"qkv_{tag}_rho"], g[f"qkv_{tag}_cos"],
                                             g[f"qkv_{tag}_sin"], g[f"qkv_{tag}_scale"], 1e-6)
    for got, name in ((q, "q"), (k, "k"), (v, "v")):
        np.testing.assert_allclose(got, g[f"qkv_{tag}_{name}"], atol=1e-12, rtol=1e-12)


@pytest.mark.parametrize("tag,max_radius", [("g075", 0.75), ("g1024", 1024.0), ("g0", 0.0)])
def test_carried_residual_gauge_matches_reference(golden, tag, max_radius):
    g = golden("ops_small.npz")
    y, r = O.carried_residual_gauge(g["res_y"], g["res_rho"], g["res_branch"], g["res_alpha"], 1e-6, 1e-6,
                                    max_radius)
    np.testing.assert_allclose(y, g[f"res_{tag}_y"], atol=1e-12, rtol=1e-12)
    np.testing.assert_allclose(r, g[f"res_{tag}_rho"], atol=1e-12, rtol=1e-12)


def test_carried_residual_equals_materialized_ngpt_residual(golden):
    # tests/test_kernels.py:16-43 of the reference: carried form == normalise((1-a) h + a normalise(b))
    g = golden("ops_small.npz")
    y, rho, b, a = g["res_y"], g["res_rho"], g["res_branch"], g["res_alpha"]
    u, rp = O.carried_residual(y, rho, b, a, 1e-9, 1e-9)
    href = O.reference_residual(y / rho[..., None], b, a, 1e-9, 1e-9)
    np.testing.assert_allclose(u / rp[..., None], href, atol=1e-10, rtol=1e-10)


@pytest.mark.parametrize("tag", ["a", "b"])
def test_causal_attention_matches_reference_sdpa(golden, tag):
    g = golden("ops_small.npz")
    q = g[f"sdpa_{tag}_q"]
    o = O.causal_attention(q, g[f"sdpa_{tag}_k"], g[f"sdpa_{tag}_v"], np.sqrt(q.shape[-1]))
    np.testing.assert_allclose(o, g[f"sdpa_{tag}_o"], atol=1e-12, rtol=1e-12)


def test_isolated_attention_cfg2_rows_match_reference(golden):
    """B=8, H=16, T=2048, Dh=64 nGPT attention (inputs from Generator(1)); selected query rows."""
    g = golden("attn_cfg2.npz")
    B, H, T, D = 8, 16, 2048, 64
    gen = torch.Generator().manual_seed(1)
    q = torch.randn(B, T, H, D, generator=gen)
    k = torch.randn(B, T, H, D, generator=gen)
    v = torch.randn(B, T, H, D, generator=gen)
    s = torch.rand(D, generator=gen) * 0.2 + 0.9
    q = (q / q.norm(dim=-1, keepdim=True) * s).numpy().astype(np.float64)
    k = (k / k.norm(dim=-1, keepdim=True) * s).numpy().astype(np.float64)
    v = v.numpy().astype(np.float64)
    rows = g["rows"]
    for b, key in ((0, "o_b0_rows"), (7, "o_b7_rows")):
        kb, vb = k[b], v[b]                     # [T, H, D]
        for i, t in enumerate(rows):
            sc = np.einsum("hd,thd->ht", q[b, t], kb[: t + 1]) * 8.0
            p = np.exp(sc - sc.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            o = np.einsum("ht,thd->hd", p, vb[: t + 1])
            np.testing.assert_allclose(o, g[key][i], atol=2e-6, rtol=0)


def test_small_model_forward_matches_reference(golden):
    """The reference's own equivalence config (tests/test_models.py:7-31), fp64."""
    g = golden("model_small.npz")
    w = {k[2:]: v for k, v in g.items() if k.startswith("w:")}
    cfg = O.OracleConfig(**SMALL)
    logits, loss, states = O.efficient_ngpt_forward(cfg, w, g["idx"], g["targets"], keep_states=True)
    # fp64 everywhere except the rotary tables, which the reference builds in fp32 with torch's
    # (1-ulp) cos/sin; the oracle's correctly rounded tables differ by <= 1 fp32 ulp.
    np.testing.assert_allclose(logits, g["logits"], atol=1e-7, rtol=1e-6)
    assert abs(loss - float(g["loss"])) < 1e-8
    for i, (y, r) in enumerate(states):
        np.testing.assert_allclose(y, g[f"y{i}"], atol=1e-7, rtol=1e-6)
        np.testing.assert_allclose(r, g[f"rho{i}"], atol=1e-7, rtol=1e-6)
    # and the reference's materialised nGPT forward agrees (tests/test_models.py:20-31 tolerance)
    np.testing.assert_allclose(logits, g["ref_logits"], atol=1e-7, rtol=1e-6)


def test_small_model_init_matches_reference(golden):
    g = golden("model_small.npz")
    torch.manual_seed(1)
    from engpt_b200 import EfficientNGPT, ModelConfig
    model = EfficientNGPT(ModelConfig(**SMALL)).double()
    sd = model.state_dict()
    ref = {k[2:]: v for k, v in g.items() if k.startswith("w:")}
    assert list(sd.keys()) == list(ref.keys())
    for k, v in sd.items():
        np.testing.assert_array_equal(v.numpy(), ref[k])


@pytest.mark.parametrize("name,cfg", [("cfg1.npz", CFG1), ("cfg4_deep.npz", CFG4), ("cfg3_d1024.npz", CFG3)])
def test_seeded_init_fingerprint_matches_reference(golden, name, cfg):
    g = golden(name)
    model = seeded_model(cfg, seed=0)
    names, fp = fingerprint(model.state_dict())
    assert list(names) == list(g["w_names"])
    np.testing.assert_array_equal(fp, g["w_fp"])


def _ids(g):
    return g["idx"].astype(np.int64), g["targets"].astype(np.int64)


def test_cfg1_fp32_forward_matches_reference(golden):
    """EfficientNGPT L=4, d=256, H=4, T=256, B=16 fp32: loss, per-row logsumexp, per-layer Y/rho."""
    g = golden("cfg1.npz")
    model = seeded_model(CFG1, seed=0)
    w = state_numpy(model)
    idx, tgt = _ids(g)
    cfg = O.OracleConfig(**CFG1)
    logits, loss, states = O.efficient_ngpt_forward(cfg, w, idx, tgt, dtype=np.float32, keep_states=True,
                                                    state_rows=[0])
    assert abs(loss - float(g["loss"])) < 1e-4
    np.testing.assert_allclose(O.row_logsumexp(logits), g["lse"], atol=2e-4, rtol=0)
    np.testing.assert_allclose(logits[0, :, :64], g["logits_b0_v64"], atol=2e-4, rtol=0)
    rows = g["state_rows"]
    for i in g["state_layers"]:
        y, r = states[i]
        h = y[0] / r[0][:, None]
        assert row_rel_err(h[rows], g[f"h{i}"]) < 1e-5
        np.testing.assert_allclose(r[0], g[f"rho{i}"], rtol=1e-4)


def test_cfg4_deep_fp32_forward_matches_reference(golden):
    """128-layer carried stack (gauge active): batch row 0, every 8th layer."""
    g = golden("cfg4_deep.npz")
    model = seeded_model(CFG4, seed=0)
    w = state_numpy(model)
    idx, tgt = _ids(g)
    cfg = O.OracleConfig(**CFG4)
    logits, _, states = O.efficient_ngpt_forward(cfg, w, idx[:1], tgt[:1], dtype=np.float32, keep_states=True)
    np.testing.assert_allclose(O.row_logsumexp(logits)[0], g["lse"][0], atol=1e-3, rtol=0)
    rows = g["state_rows"]
    for i in g["state_layers"]:
        y, r = states[i]
        assert np.isfinite(y).all() and np.isfinite(r).all()
        assert row_rel_err(y[0, rows] / r[0, rows][:, None], g[f"h{i}"]) < 1e-4
        assert float(r.max()) <= 1024.0 * (1 + 1e-6)
    assert float(g["rhomax8"]) == pytest.approx(1024.0)


def test_oracle_sphere_ops_match_reference(golden):
    """Retraction and tangent projection (engpt/kernels.py:98-136) of the oracle vs the reference's outputs."""
    g = golden("sphere_small.npz")
    for tag in ("a", "b", "c"):
        w, gr = g[f"sph_{tag}_w"], g[f"sph_{tag}_g"]
        np.testing.assert_allclose(O.normalize_rows(w, 1e-6), g[f"sph_{tag}_rows"], rtol=1e-13, atol=1e-15)
        np.testing.assert_allclose(O.normalize_columns(w, 1e-6), g[f"sph_{tag}_cols"], rtol=1e-13, atol=1e-15)
        np.testing.assert_allclose(O.project_row_grad(g[f"sph_{tag}_wr"], gr), g[f"sph_{tag}_prow"], rtol=1e-12,
                                   atol=1e-13)
        np.testing.assert_allclose(O.project_column_grad(g[f"sph_{tag}_wc"], gr), g[f"sph_{tag}_pcol"], rtol=1e-12,
                                   atol=1e-13)


def test_optimizer_step_host_logic_matches_reference_on_cpu(golden):
    """engpt_b200.optim.NGPTAdamW on CPU parameters (its PyTorch expressions, the reference's CPU path) reproduces
    the reference's NGPTAdamW step (engpt/optim.py:38-67) from the same seeded weights and gradients."""
    from engpt_b200 import EfficientNGPT, ModelConfig
    from engpt_b200.optim import NGPTAdamW
    g = golden("optim_step.npz")
    cfg = ModelConfig(vocab_size=64, block_size=16, n_layer=2, n_head=2, n_embd=32, mlp_ratio=2.0, dropout=0.0)
    torch.manual_seed(2)
    model = EfficientNGPT(cfg)
    for n, p in model.named_parameters():
        p.grad = torch.as_tensor(g["g:" + n]).clone()
    NGPTAdamW(model, lr=1e-2).step()
    for n, p in model.named_parameters():
        np.testing.assert_allclose(p.detach().numpy(), g["w:" + n], rtol=1e-6, atol=1e-7)
