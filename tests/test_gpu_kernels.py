"""Op-level parity of the CUDA kernels against the oracle and the reference's golden vectors (B200)."""

import math

import numpy as np
import pytest
import torch

from engpt_b200 import _lib, kernels as K
from oracle import ngpt_oracle as O

pytestmark = pytest.mark.gpu


def t(x, dev, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(x)).to(device=dev, dtype=dtype)


def bf16_round(x):
    return torch.as_tensor(np.asarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy().astype(np.float64)


@pytest.fixture(autouse=True)
def _no_grad_and_clean_status(cuda):
    _lib.clear_device_status()
    with torch.no_grad():
        yield
    assert _lib.device_status() == 0, "a kernel recorded a device-side failure"


def test_rotary_tables_match_reference(golden, cuda):
    g = golden("ops_small.npz")
    cos, sin = K.rotary_frequencies(2048, 64, device=cuda, dtype=torch.float32, theta=10000.0)
    np.testing.assert_allclose(cos.cpu().numpy(), g["rope2048_cos"], atol=2.5e-7, rtol=0)
    np.testing.assert_allclose(sin.cpu().numpy(), g["rope2048_sin"], atol=2.5e-7, rtol=0)


@pytest.mark.parametrize("tag", ["even", "odd"])
def test_qkv_postprocess_fp32_matches_reference(golden, cuda, tag):
    g = golden("ops_small.npz")
    q, k, v = K.qkv_postprocess_from_carried(t(g[f"qkv_{tag}_in"], cuda), t(g[f"qkv_{tag}_rho"], cuda),
                                             t(g[f"qkv_{tag}_cos"], cuda), t(g[f"qkv_{tag}_sin"], cuda),
                                             t(g[f"qkv_{tag}_scale"], cuda), 1e-6)
    for got, name in ((q, "q"), (k, "k"), (v, "v")):
        np.testing.assert_allclose(got.cpu().numpy(), g[f"qkv_{tag}_{name}"], atol=2e-6, rtol=2e-6)


@pytest.mark.parametrize("dh", [64, 128, 16, 48])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_qkv_postprocess_layouts_vs_oracle(cuda, dh, dtype):
    rng = np.random.default_rng(dh)
    B, T, H = 2, 37, 3
    qkv = rng.standard_normal((B, T, 3, H, dh)) * 3.0
    qkv[1, 5, 0, 2] *= 1e-9  # exercise the rho * eps guard
    rho = rng.uniform(0.2, 900.0, (B, T))
    cos, sin = O.rotary_frequencies(T, dh, 10000.0)
    scale = rng.uniform(0.9, 1.1, (H, dh))
    qkv_dev = t(qkv, cuda, dtype)
    qkv_in = qkv_dev.float().cpu().numpy().astype(np.float64)
    ref = O.qkv_postprocess_from_carried(qkv_in, rho.astype(np.float32).astype(np.float64), cos.astype(np.float64),
                                         sin.astype(np.float64), scale.astype(np.float32).astype(np.float64), 1e-6)
    tol = 2e-6 if dtype == torch.float32 else 1e-2
    q, k, v = K.qkv_postprocess_from_carried(qkv_dev, t(rho, cuda), t(cos, cuda), t(sin, cuda), t(scale, cuda), 1e-6)
    for got, exp in zip((q, k, v), ref):
        np.testing.assert_allclose(got.float().cpu().numpy(), exp, atol=tol * np.abs(exp).max(), rtol=tol)
    # head-major layout written directly for the attention kernel
    hm = [torch.empty(B, H, T, dh, device=cuda, dtype=dtype) for _ in range(3)]
    K.qkv_postprocess_into(qkv_dev, t(rho, cuda), t(cos, cuda), t(sin, cuda), t(scale, cuda), 1.0, 1e-6,
                           *hm, head_major=True)
    for got, exp in zip(hm, ref):
        np.testing.assert_allclose(got.transpose(1, 2).float().cpu().numpy(), exp, atol=tol * np.abs(exp).max(),
                                   rtol=tol)


@pytest.mark.parametrize("dh,H", [(64, 16), (128, 4), (16, 2)])
def test_qkv_postprocess_in_place_vs_oracle(cuda, dh, H):
    """q, k, v written back over the [B, T, 3, H, Dh] projection (the engine's layout)."""
    rng = np.random.default_rng(dh + H)
    B, T = 2, 45
    qkv = rng.standard_normal((B, T, 3, H, dh)) * 2.0
    rho = rng.uniform(0.5, 600.0, (B, T))
    cos, sin = O.rotary_frequencies(T, dh, 10000.0)
    scale = rng.uniform(0.9, 1.1, (H, dh))
    buf = t(qkv, cuda, torch.bfloat16)
    ref = O.qkv_postprocess_from_carried(buf.float().cpu().numpy().astype(np.float64),
                                         rho.astype(np.float32).astype(np.float64), cos.astype(np.float64),
                                         sin.astype(np.float64), scale.astype(np.float32).astype(np.float64), 1e-6)
    rho_d, cos_d, sin_d, sc_d = t(rho, cuda), t(cos, cuda), t(sin, cuda), t(scale, cuda)
    _lib.call("engpt_qkv_postprocess", buf.data_ptr(), _lib.BF16, rho_d.data_ptr(), cos_d.data_ptr(),
              sin_d.data_ptr(), dh // 2, sc_d.data_ptr(), 1.0, 1e-6, B, T, H, dh, None, None, None,
              _lib.QKV_INPLACE, _lib.stream_handle(cuda))
    got = buf.float().cpu().numpy()
    for s_idx in range(3):
        exp = ref[s_idx]
        np.testing.assert_allclose(got[:, :, s_idx], exp, atol=1e-2 * np.abs(exp).max(), rtol=1e-2)


@pytest.mark.parametrize("tag,max_radius", [("g075", 0.75), ("g1024", 1024.0), ("g0", 0.0)])
def test_carried_residual_gauge_fp32_matches_reference(golden, cuda, tag, max_radius):
    g = golden("ops_small.npz")
    y, r = K.carried_residual_gauge(t(g["res_y"], cuda), t(g["res_rho"], cuda), t(g["res_branch"], cuda),
                                    t(g["res_alpha"], cuda), 1e-6, 1e-6, max_radius)
    np.testing.assert_allclose(y.cpu().numpy(), g[f"res_{tag}_y"], rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(r.cpu().numpy(), g[f"res_{tag}_rho"], rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("d,rows", [(32, 77), (100, 77), (256, 77), (1024, 77), (2048, 77), (4096, 77),
                                    (256, 20000), (1024, 20000), (2048, 20000)])
@pytest.mark.parametrize("bdtype", [torch.float32, torch.bfloat16])
def test_carried_residual_aux_outputs_and_in_place(cuda, d, rows, bdtype):
    """Against the oracle, in place, every aux mode.  77 rows take the four-warps-per-row kernel (d a multiple of
    8, up to 2048) or the generic one; 20000 rows the one-warp-per-row kernel."""
    rng = np.random.default_rng(d + rows)
    y = rng.standard_normal((rows, d)) * 40.0
    rho = rng.uniform(1.0, 1000.0, rows)
    branch = rng.standard_normal((rows, d))
    branch[3] = 0.0
    alpha = rng.uniform(-0.1, 0.1, d)
    b_dev = t(branch, cuda, bdtype)
    b_in = b_dev.float().cpu().numpy().astype(np.float64)
    a32 = alpha.astype(np.float32).astype(np.float64)
    mult = 1.6
    eff = (np.abs(a32) * mult).astype(np.float32).astype(np.float64)
    y32 = y.astype(np.float32).astype(np.float64)
    r32 = rho.astype(np.float32).astype(np.float64)
    ey, er = O.carried_residual_gauge(y32, r32, b_in, eff, 1e-6, 1e-6, 1024.0)
    for mode in (_lib.AUX_NONE, _lib.AUX_BF16_Y, _lib.AUX_BF16_H, _lib.AUX_F32_H):
        yd, rd = t(y, cuda), t(rho, cuda)
        aux = None
        if mode in (_lib.AUX_BF16_Y, _lib.AUX_BF16_H):
            aux = torch.empty(rows, d, device=cuda, dtype=torch.bfloat16)
        elif mode == _lib.AUX_F32_H:
            aux = torch.empty(rows, d, device=cuda, dtype=torch.float32)
        K.carried_residual_into(yd, rd, b_dev, t(alpha, cuda), mult, True, 1e-6, 1e-6, 1024.0, yd, rd, aux, mode)
        np.testing.assert_allclose(yd.cpu().numpy(), ey, rtol=1e-5, atol=1e-5 * np.abs(ey).max())
        np.testing.assert_allclose(rd.cpu().numpy(), er, rtol=1e-5)
        if mode == _lib.AUX_BF16_Y:
            np.testing.assert_allclose(aux.float().cpu().numpy(), ey, rtol=8e-3, atol=1e-3 * np.abs(ey).max())
        elif mode in (_lib.AUX_BF16_H, _lib.AUX_F32_H):
            h = ey / er[:, None]
            tol = 8e-3 if mode == _lib.AUX_BF16_H else 1e-5
            np.testing.assert_allclose(aux.float().cpu().numpy(), h, rtol=tol, atol=tol * np.abs(h).max())
    assert float(er.max()) <= 1024.0 * (1 + 1e-6)


def _attn_inputs(B, T, H, D, seed, normalize=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, D, generator=g)
    k = torch.randn(B, T, H, D, generator=g)
    v = torch.randn(B, T, H, D, generator=g)
    if normalize:
        s = torch.rand(D, generator=g) * 0.2 + 0.9
        q = q / q.norm(dim=-1, keepdim=True) * s
        k = k / k.norm(dim=-1, keepdim=True) * s
    return q, k, v


@pytest.mark.parametrize("tag", ["a", "b"])
def test_attention_simt_fp32_matches_reference(golden, cuda, tag):
    g = golden("ops_small.npz")
    q = g[f"sdpa_{tag}_q"]
    o = K.causal_sdpa(t(q, cuda), t(g[f"sdpa_{tag}_k"], cuda), t(g[f"sdpa_{tag}_v"], cuda),
                      scale=math.sqrt(q.shape[-1]), dropout_p=0.0)
    np.testing.assert_allclose(o.cpu().numpy(), g[f"sdpa_{tag}_o"], atol=2e-6, rtol=2e-5)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("T", [1, 100, 128, 130, 256, 333, 1024])
def test_attention_tcgen05_bf16_vs_oracle(cuda, D, T):
    B, H = 2, 3
    q, k, v = _attn_inputs(B, T, H, D, seed=T + D)
    qb, kb, vb = (x.to(cuda, torch.bfloat16) for x in (q, k, v))
    o = K.causal_sdpa(qb, kb, vb, scale=math.sqrt(D), dropout_p=0.0, impl="tcgen05")
    ref = O.causal_attention(*(x.float().cpu().numpy().astype(np.float64) for x in (qb, kb, vb)), math.sqrt(D))
    err = np.abs(o.float().cpu().numpy() - ref).max()
    # bf16 P and bf16 output rounding: compare with torch's own bf16 SDPA on the same inputs
    sd = torch.nn.functional.scaled_dot_product_attention(qb.transpose(1, 2), kb.transpose(1, 2),
                                                          vb.transpose(1, 2), is_causal=True,
                                                          scale=math.sqrt(D)).transpose(1, 2)
    err_torch = np.abs(sd.float().cpu().numpy() - ref).max()
    assert err < 1.5e-2, (err, err_torch)
    assert err <= 2.0 * err_torch + 2e-3, (err, err_torch)


@pytest.mark.parametrize("B,T,H", [(8, 1152, 16), (8, 1200, 16), (2, 2048, 16), (20, 2048, 16)])
def test_attention_tcgen05_many_bands_per_cta(cuda, B, T, H):
    """More 256-query bands than SMs, so every CTA of the persistent head_dim-64 kernel walks several bands:
    the Q double buffer, the job / K-V / PV counters that run across bands, the band store deferred past the
    next band's first job, last bands whose second 128-row tile is empty (T = 1152: T mod 256 = 128) or only
    partly filled (T = 1200: T mod 256 = 176).  The first three take the bands by size class (their K/V fit
    in L2), B=20 by (batch, head).  Reference: torch's fp32 causal SDPA on the same bf16-rounded inputs;
    bound as in the oracle test above."""
    D = 64
    q, k, v = _attn_inputs(B, T, H, D, seed=B * T + H)
    qb, kb, vb = (x.to(cuda, torch.bfloat16) for x in (q, k, v))
    o = K.causal_sdpa(qb, kb, vb, scale=math.sqrt(D), dropout_p=0.0, impl="tcgen05")

    def sdpa(x, y, z):
        return torch.nn.functional.scaled_dot_product_attention(
            x.transpose(1, 2), y.transpose(1, 2), z.transpose(1, 2), is_causal=True, scale=math.sqrt(D)
        ).transpose(1, 2)

    ref = sdpa(qb.float(), kb.float(), vb.float())
    err = (o.float() - ref).abs().max().item()
    err_torch = (sdpa(qb, kb, vb).float() - ref).abs().max().item()
    assert err < 1.5e-2, (err, err_torch)
    assert err <= 2.0 * err_torch + 2e-3, (err, err_torch)


def _ngpt_inputs(B, T, H, D, s_heads, seed):
    """Unit q/k per head times an effective scale s[h, :] (the QKV post-process output), v ~ N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, T, H, D, generator=g) for _ in range(3))
    s = torch.stack([torch.rand(D, generator=g) * 0.2 + (sh - 0.1) for sh in s_heads])    # [H, D]
    q = q / q.norm(dim=-1, keepdim=True) * s
    k = k / k.norm(dim=-1, keepdim=True) * s
    return q, k, v, s


def _ngpt_attention(cuda, qb, kb, vb, s_raw, mult, scale):
    B, T, H, D = qb.shape
    o = torch.empty_like(qb)
    strides = K.attention_strides(qb, kb, vb, o, head_major=False)
    s_dev = s_raw.to(cuda, torch.float32).contiguous()
    _lib.call("engpt_ngpt_attention", qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), o.data_ptr(), _lib.BF16, B, T, H,
              D, float(scale), strides.data_ptr(), s_dev.data_ptr(), float(mult), _stream())
    return o


@pytest.mark.parametrize("B,T,H,D", [(2, 1, 3, 64), (2, 100, 3, 64), (2, 128, 3, 64), (1, 130, 2, 64), (2, 333, 3, 64),
                                     (2, 1024, 4, 64), (8, 1200, 16, 64), (4, 2048, 16, 64), (2, 1, 2, 128),
                                     (2, 333, 3, 128), (1, 2048, 4, 128)])
def test_ngpt_attention_fixed_offset_vs_oracle(cuda, B, T, H, D):
    """The tcgen05 kernels (head_dim 64 and 128) with the softmax offset taken from the per-head score bound (no
    running max), against the fp64 oracle on the same bf16 inputs: within torch's own bf16 SDPA error, as the
    general kernels."""
    q, k, v, s = _ngpt_inputs(B, T, H, D, [1.0] * H, seed=B * T + H)
    qb, kb, vb = (x.to(cuda, torch.bfloat16) for x in (q, k, v))
    scale = math.sqrt(D)
    o = _ngpt_attention(cuda, qb, kb, vb, s / 32.0, 32.0, scale)       # raw parameter x multiplier
    ref = O.causal_attention(*(x.float().cpu().numpy().astype(np.float64) for x in (qb, kb, vb)), scale)
    err = np.abs(o.float().cpu().numpy() - ref).max()
    sd = torch.nn.functional.scaled_dot_product_attention(qb.transpose(1, 2), kb.transpose(1, 2),
                                                          vb.transpose(1, 2), is_causal=True,
                                                          scale=scale).transpose(1, 2)
    err_torch = np.abs(sd.float().cpu().numpy() - ref).max()
    assert err < 1.5e-2, (err, err_torch)
    assert err <= 2.0 * err_torch + 2e-3, (err, err_torch)


def test_ngpt_attention_mixed_heads_take_both_softmax_paths(cuda):
    """Heads whose bound is small (fixed offset) and large (s = 3: 8 log2(e) 9 > 48, running max) in one launch,
    several bands per CTA: both paths against the oracle, per head within twice torch's own bf16 SDPA error (the
    s = 3 heads are nearly one-hot, where bf16 rounding of the inputs dominates)."""
    B, T, H, D = 4, 1536, 8, 64
    q, k, v, s = _ngpt_inputs(B, T, H, D, [1.0, 3.0, 0.5, 1.0, 3.0, 1.0, 2.2, 1.0], seed=17)
    qb, kb, vb = (x.to(cuda, torch.bfloat16) for x in (q, k, v))
    o = _ngpt_attention(cuda, qb, kb, vb, s, 1.0, 8.0)
    ref = O.causal_attention(*(x.float().cpu().numpy().astype(np.float64) for x in (qb, kb, vb)), 8.0)
    sd = torch.nn.functional.scaled_dot_product_attention(qb.transpose(1, 2), kb.transpose(1, 2),
                                                          vb.transpose(1, 2), is_causal=True,
                                                          scale=8.0).transpose(1, 2).float().cpu().numpy()
    got = o.float().cpu().numpy()
    for h in range(H):
        err = np.abs(got[:, :, h] - ref[:, :, h]).max()
        err_torch = np.abs(sd[:, :, h] - ref[:, :, h]).max()
        assert err <= 2.0 * err_torch + 2e-3, (h, err, err_torch)


def test_ngpt_attention_isolated_cfg2(golden, cuda):
    """The isolated attention configuration (B=8, H=16, T=2048, Dh=64, s ~ U(0.9, 1.1)) through the fixed-offset
    kernel against the reference's golden rows."""
    g = golden("attn_cfg2.npz")
    B, H, T, D = 8, 16, 2048, 64
    gen = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(B, T, H, D, generator=gen) for _ in range(3))
    s = torch.rand(D, generator=gen) * 0.2 + 0.9
    q = q / q.norm(dim=-1, keepdim=True) * s
    k = k / k.norm(dim=-1, keepdim=True) * s
    o = _ngpt_attention(cuda, *(x.to(cuda, torch.bfloat16) for x in (q, k, v)), s.expand(H, D), 1.0, 8.0)
    rows = g["rows"]
    np.testing.assert_allclose(o[0, rows].float().cpu().numpy(), g["o_b0_rows"], atol=1.5e-2)
    np.testing.assert_allclose(o[7, rows].float().cpu().numpy(), g["o_b7_rows"], atol=1.5e-2)
    assert abs(o.double().abs().sum().item() - float(g["o_abs_sum"])) / float(g["o_abs_sum"]) < 5e-3


@pytest.mark.parametrize("D", [64, 128])
def test_attention_tcgen05_head_major_strides_and_unnormalised_inputs(cuda, D):
    # general (not unit-norm) q/k exercise the reference-max raising path; head-major strides exercise TMA maps
    B, T, H = 1, 520, 2
    q, k, v = _attn_inputs(B, T, H, D, seed=7, normalize=False)
    q = q * 3.0
    qh, kh, vh = (x.transpose(1, 2).contiguous().to(cuda, torch.bfloat16) for x in (q, k, v))  # [B,H,T,D]
    o = torch.empty(B, T, H, D, device=cuda, dtype=torch.bfloat16)
    strides = K.attention_strides(qh, kh, vh, o, head_major=True)
    strides[9:] = torch.tensor([o.stride(0), o.stride(1), o.stride(2)])
    K.causal_attention_into(qh, kh, vh, o, 0.5, strides, B, T, H, D, _lib.ATTN_TCGEN05)
    ref = O.causal_attention(*(x.transpose(1, 2).float().cpu().numpy().astype(np.float64) for x in (qh, kh, vh)),
                             0.5)
    np.testing.assert_allclose(o.float().cpu().numpy(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("T", [130, 700])
def test_attention_tcgen05_one_tile_variant_vs_oracle(cuda, T):
    """The one-128-query-tile-per-CTA kernel (head_dim 64 comparison path)."""
    q, k, v = _attn_inputs(2, T, 2, 64, seed=T)
    qb, kb, vb = (x.to(cuda, torch.bfloat16) for x in (q, k, v))
    o = K.causal_sdpa(qb, kb, vb, scale=8.0, dropout_p=0.0, impl="tcgen05_1tile")
    ref = O.causal_attention(*(x.float().cpu().numpy().astype(np.float64) for x in (qb, kb, vb)), 8.0)
    assert np.abs(o.float().cpu().numpy() - ref).max() < 1.5e-2


@pytest.mark.parametrize("D", [64, 128])
def test_attention_tcgen05_score_jumps(cuda, D):
    """Scores that jump far above the running reference max mid-sequence (exercises the O/P rescale
    and the tile-restart paths of the kernel): keys at a few positions are large multiples of a query."""
    B, T, H = 1, 600, 2
    q, k, v = _attn_inputs(B, T, H, D, seed=99, normalize=False)
    for pos, mult in ((5, 4.0), (300, 30.0), (450, 200.0)):
        k[:, pos] = q[:, pos + 3] * mult
    qb, kb, vb = (x.to(cuda, torch.bfloat16) for x in (q, k, v))
    scale = 1.0 / math.sqrt(D)
    o = K.causal_sdpa(qb, kb, vb, scale=scale, dropout_p=0.0, impl="tcgen05")
    ref = O.causal_attention(*(x.float().cpu().numpy().astype(np.float64) for x in (qb, kb, vb)), scale)
    assert np.isfinite(o.float().cpu().numpy()).all()
    np.testing.assert_allclose(o.float().cpu().numpy(), ref, atol=2e-2, rtol=2e-2)


def test_attention_simt_bf16_odd_head_dim(cuda):
    q, k, v = _attn_inputs(2, 77, 2, 24, seed=3)
    qb, kb, vb = (x.to(cuda, torch.bfloat16) for x in (q, k, v))
    o = K.causal_sdpa(qb, kb, vb, scale=math.sqrt(24), dropout_p=0.0)
    ref = O.causal_attention(*(x.float().cpu().numpy().astype(np.float64) for x in (qb, kb, vb)), math.sqrt(24))
    np.testing.assert_allclose(o.float().cpu().numpy(), ref, atol=1e-2, rtol=1e-2)


def test_isolated_attention_cfg2(golden, cuda):
    """B=8, H=16, T=2048, Dh=64 nGPT attention, bf16 (and fp32 on the CUDA-core path)."""
    g = golden("attn_cfg2.npz")
    B, H, T, D = 8, 16, 2048, 64
    q, k, v = _attn_inputs(B, T, H, D, seed=1)
    rows = g["rows"]
    ob = K.causal_sdpa(*(x.to(cuda, torch.bfloat16) for x in (q, k, v)), scale=8.0, dropout_p=0.0)
    np.testing.assert_allclose(ob[0, rows].float().cpu().numpy(), g["o_b0_rows"], atol=1.5e-2)
    np.testing.assert_allclose(ob[7, rows].float().cpu().numpy(), g["o_b7_rows"], atol=1.5e-2)
    abs_sum = ob.double().abs().sum().item()
    assert abs(abs_sum - float(g["o_abs_sum"])) / float(g["o_abs_sum"]) < 5e-3
    of = K.causal_sdpa(*(x.to(cuda) for x in (q, k, v)), scale=8.0, dropout_p=0.0)
    np.testing.assert_allclose(of[0, rows].cpu().numpy(), g["o_b0_rows"], atol=2e-5)
    assert abs(of.double().sum().item() - float(g["o_sum"])) < 1e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_swiglu_vs_oracle(cuda, dtype):
    rng = np.random.default_rng(5)
    rows, W = 33, 264
    ug = rng.standard_normal((rows, 2 * W))
    su, sg = rng.uniform(0.5, 1.5, W), rng.uniform(0.5, 1.5, W)
    ug_dev = t(ug, cuda, dtype)
    out = torch.empty(rows, W, device=cuda, dtype=dtype)
    K.swiglu_into(ug_dev, t(su, cuda), t(sg, cuda), 16.0, 16.0, out)
    x = ug_dev.float().cpu().numpy().astype(np.float64)
    u = x[:, :W] * su.astype(np.float32) * 16.0
    gg = x[:, W:] * sg.astype(np.float32) * 16.0
    exp = u * O.silu(gg)
    tol = 1e-5 if dtype == torch.float32 else 8e-3
    np.testing.assert_allclose(out.float().cpu().numpy(), exp, rtol=tol, atol=tol * np.abs(exp).max())


def test_cast_f32_bf16_many_matches_torch(cuda):
    import ctypes
    g = torch.Generator().manual_seed(3)
    srcs = [torch.randn(n, generator=g).to(cuda) for n in (1, 7, 8, 1000, 4096 * 3 + 5)]
    srcs.append(torch.randn(64, 70, generator=g).to(cuda)[:, 3:67].contiguous())
    dsts = [torch.empty(x.shape, device=cuda, dtype=torch.bfloat16) for x in srcs]
    n = len(srcs)
    _lib.call("engpt_cast_f32_bf16_many", (ctypes.c_void_p * n)(*[x.data_ptr() for x in srcs]),
              (ctypes.c_void_p * n)(*[x.data_ptr() for x in dsts]),
              (ctypes.c_int64 * n)(*[x.numel() for x in srcs]), n, _lib.stream_handle(cuda))
    for x, y in zip(srcs, dsts):
        assert torch.equal(y, x.to(torch.bfloat16))


def test_cast_f32_bf16_many_batches_and_sizes(cuda):
    """More tensors than one launch takes (64), an empty one, and sizes from 1 element to 2M (blocks are handed
    out in proportion to the sizes)."""
    import ctypes
    g = torch.Generator().manual_seed(5)
    sizes = [0, 3, 2_000_001] + [(i * 7919) % 40000 + 1 for i in range(67)]
    srcs = [torch.randn(n, generator=g).to(cuda) for n in sizes]
    dsts = [torch.full(x.shape, 7.0, device=cuda, dtype=torch.bfloat16) for x in srcs]
    n = len(srcs)
    _lib.call("engpt_cast_f32_bf16_many", (ctypes.c_void_p * n)(*[x.data_ptr() for x in srcs]),
              (ctypes.c_void_p * n)(*[x.data_ptr() for x in dsts]),
              (ctypes.c_int64 * n)(*[x.numel() for x in srcs]), n, _lib.stream_handle(cuda))
    for x, y in zip(srcs, dsts):
        assert torch.equal(y, x.to(torch.bfloat16))


@pytest.mark.parametrize("V", [1001, 50257])
def test_cross_entropy_vs_oracle(cuda, V):
    from engpt_b200 import EfficientNGPT
    rng = np.random.default_rng(V)
    rows = 37
    logits = torch.as_tensor(rng.standard_normal((rows, V)) * 4.0).to(cuda, torch.bfloat16)
    tgt = rng.integers(0, V, rows)
    tgt[5] = -100
    loss = EfficientNGPT.loss_from_logits(logits.view(1, rows, V), torch.as_tensor(tgt).view(1, rows).to(cuda))
    x = logits.float().cpu().numpy().astype(np.float64)
    keep = tgt != -100
    exp = O.cross_entropy(x[keep][None], tgt[keep][None])
    assert abs(loss.item() - exp) < 1e-4


# ------------------------------------------------------------ tcgen05 GEMM and fused projections
def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 520, 200), (1000, 3072, 1024), (4096, 1024, 4096)])
def test_gemm_bf16_matches_fp32_reference(cuda, M, N, K):
    """C = A B^T (F.linear): ragged M / N / K exercise TMA out-of-bounds fill and the masked epilogue."""
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(cuda, torch.bfloat16)
    b = torch.randn(N, K, generator=g).to(cuda, torch.bfloat16)
    c = torch.full((M, N), float("nan"), device=cuda, dtype=torch.bfloat16)
    _lib.call("engpt_gemm_bf16", a.data_ptr(), K, b.data_ptr(), K, c.data_ptr(), N, M, N, K, _stream())
    ref = a.float() @ b.float().t()
    err = ((c.float() - ref).abs().max() / ref.abs().max()).item()
    assert err < 8e-3, err   # bf16 output rounding (2^-8 relative)


@pytest.mark.parametrize("rows", [200, 4096])
def test_up_gate_swiglu_matches_unfused_path(cuda, rows):
    """Fused up/gate GEMM + SwiGLU vs cuBLAS GEMM + the SwiGLU kernel (engpt/kernels.py:182-206)."""
    d, W = 256, 512
    g = torch.Generator().manual_seed(rows)
    x = (torch.randn(rows, d, generator=g) * 0.5).to(cuda, torch.bfloat16)
    w = (torch.randn(2 * W, d, generator=g) / 16).to(cuda, torch.bfloat16)
    su = (torch.rand(W, generator=g) + 0.5).to(cuda)
    sg = (torch.rand(W, generator=g) + 0.5).to(cuda)
    fused = torch.empty(rows, W, device=cuda, dtype=torch.bfloat16)
    _lib.call("engpt_up_gate_swiglu", x.data_ptr(), w.data_ptr(), su.data_ptr(), sg.data_ptr(), 16.0, 16.0, rows, d,
              W, fused.data_ptr(), _stream())
    # fp32 restatement of the epilogue on the fp32 product
    ug = x.float() @ w.float().t()
    u, gate = ug[:, :W] * su * 16.0, ug[:, W:] * sg * 16.0
    ref = u * torch.nn.functional.silu(gate)
    err = ((fused.float() - ref).abs().max() / ref.abs().max()).item()
    assert err < 1e-2, err
    # and against the production unfused path (bf16 projection, then the SwiGLU kernel)
    ugb = torch.mm(x, w.t())
    hid = torch.empty_like(fused)
    _lib.call("engpt_swiglu", ugb.data_ptr(), _lib.BF16, su.data_ptr(), sg.data_ptr(), 16.0, 16.0, rows, W,
              hid.data_ptr(), _lib.BF16, _stream())
    assert ((fused.float() - hid.float()).abs().max() / hid.float().abs().max()).item() < 2e-2


@pytest.mark.parametrize("B,T", [(1, 130), (2, 256)])
def test_qkv_projection_matches_unfused_path(cuda, B, T):
    """Fused QKV GEMM + post-process vs cuBLAS GEMM + engpt_qkv_postprocess in place."""
    H, Dh = 4, 64
    d = H * Dh
    n = B * T
    g = torch.Generator().manual_seed(T)
    x = (torch.randn(n, d, generator=g) * 0.5).to(cuda, torch.bfloat16)
    w = (torch.randn(3 * d, d, generator=g) / 16).to(cuda, torch.bfloat16)
    rho = (torch.rand(n, generator=g) + 0.5).to(cuda)
    cos, sin = K.rotary_frequencies(T, Dh, device=cuda, dtype=torch.float32, theta=10000.0)
    qks = (torch.rand(H, Dh, generator=g) + 0.5).to(cuda)
    fused = torch.empty(n, 3 * d, device=cuda, dtype=torch.bfloat16)
    _lib.call("engpt_qkv_projection", x.data_ptr(), d, w.data_ptr(), rho.data_ptr(), cos.data_ptr(), sin.data_ptr(),
              Dh // 2, qks.data_ptr(), 2.0, 1e-6, B, T, H, Dh, fused.data_ptr(), _stream())
    unf = torch.mm(x, w.t())
    _lib.call("engpt_qkv_postprocess", unf.data_ptr(), _lib.BF16, rho.data_ptr(), cos.data_ptr(), sin.data_ptr(),
              Dh // 2, qks.data_ptr(), 2.0, 1e-6, B, T, H, Dh, None, None, None, _lib.QKV_INPLACE, _stream())
    diff = (fused.float() - unf.float()).abs().max().item()
    assert diff <= 2e-2 * unf.float().abs().max().item(), diff


@pytest.mark.parametrize("B,T,H,Dh", [(2, 2048, 16, 64), (1, 300, 16, 64), (1, 1024, 8, 128), (2, 130, 4, 128)])
def test_qkv_projection_vs_oracle_d1024(cuda, B, T, H, Dh):
    """Fused QKV GEMM + post-process against the fp64 oracle (engpt/kernels.py:139-179 on the exact product of
    the bf16 operands) at the benchmarked width (d=1024, H=16, Dh=64) and with head_dim 128 (the long-context
    configuration's heads): every q/k/v row within bf16 output rounding, 8e-3 of its norm."""
    d = H * Dh
    n = B * T
    g = torch.Generator().manual_seed(B * T)
    x = torch.nn.functional.normalize(torch.randn(n, d, generator=g), dim=-1).to(cuda, torch.bfloat16)
    w = torch.nn.functional.normalize(torch.randn(3 * d, d, generator=g), dim=-1).to(cuda, torch.bfloat16)
    rho = (torch.rand(n, generator=g) * 40 + 0.5).to(cuda)
    cos, sin = K.rotary_frequencies(T, Dh, device=cuda, dtype=torch.float32, theta=10000.0)
    s_qk = (torch.rand(H, Dh, generator=g) * 0.2 + 0.9) / 32.0      # raw parameter; x 32 = effective
    s_qk = s_qk.to(cuda)
    out = torch.empty(n, 3 * d, device=cuda, dtype=torch.bfloat16)
    _lib.call("engpt_qkv_projection", x.data_ptr(), d, w.data_ptr(), rho.data_ptr(), cos.data_ptr(), sin.data_ptr(),
              Dh // 2, s_qk.data_ptr(), 32.0, 1e-6, B, T, H, Dh, out.data_ptr(), _stream())
    x64 = x.double().cpu().numpy()
    w64 = w.double().cpu().numpy()
    raw = (x64 @ w64.T).reshape(B, T, 3, H, Dh)
    eff = (s_qk.cpu() * 32.0).numpy().astype(np.float64)
    ref = O.qkv_postprocess_from_carried(raw, rho.cpu().numpy().astype(np.float64).reshape(B, T),
                                         cos.cpu().numpy().astype(np.float64), sin.cpu().numpy().astype(np.float64),
                                         eff, 1e-6)
    got = out.float().cpu().numpy().reshape(B, T, 3, H, Dh)
    for i in range(3):
        err = row_rel(got[:, :, i].reshape(-1, Dh), ref[i].reshape(-1, Dh))
        assert err < 8e-3, (i, err)


def row_rel(a, b):
    num = np.sqrt(((np.asarray(a, np.float64) - b) ** 2).sum(-1))
    return float((num / np.maximum(np.sqrt((b ** 2).sum(-1)), 1e-30)).max())


def _residual_case(cuda, rows, d, K, seed):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(rows, K, generator=g) * 0.5).to(cuda, torch.bfloat16)
    w = (torch.randn(d, K, generator=g) / K ** 0.5).to(cuda, torch.bfloat16)
    y = torch.randn(rows, d, generator=g).to(cuda)
    rho = (torch.rand(rows, generator=g) * 3 + 0.25).to(cuda)
    alpha = (torch.rand(d, generator=g) - 0.3).to(cuda)     # some negative: alpha_abs folds them
    return a, w, y, rho, alpha


@pytest.mark.parametrize("rows,d,K,aux_mode", [(200, 256, 256, 2), (1000, 512, 1024, 1), (300, 1024, 1024, 2),
                                               (4224, 1024, 4096, 1), (129, 768, 512, 0)])
def test_gemm_carried_residual_matches_unfused_path(cuda, rows, d, K, aux_mode):
    """GEMM + carried residual in one kernel (clusters of d/256 CTAs) vs the GEMM, then engpt_carried_residual_gauge
    (engpt/kernels.py:277-324) on its bf16 output."""
    a, w, y, rho, alpha = _residual_case(cuda, rows, d, K, rows + d)
    branch = torch.mm(a, w.t())
    # max radius = the median ungauged rho+, so the gauge is active on about half of the rows
    y0, r0 = torch.empty_like(y), torch.empty_like(rho)
    _lib.call("engpt_carried_residual_gauge", y.data_ptr(), rho.data_ptr(), branch.data_ptr(), _lib.BF16,
              alpha.data_ptr(), 0.7, 1, 1e-6, 1e-6, 0.0, rows, d, y0.data_ptr(), r0.data_ptr(), None, 0, _stream())
    max_radius = r0.median().item()
    args = (alpha.data_ptr(), 0.7, 1, 1e-6, 1e-6, max_radius, rows, d)
    yo = torch.empty_like(y)
    ro = torch.empty_like(rho)
    aux = torch.empty(rows, d, device=cuda, dtype=torch.bfloat16)
    _lib.call("engpt_gemm_carried_residual", a.data_ptr(), K, w.data_ptr(), K, K, y.data_ptr(), rho.data_ptr(), *args,
              yo.data_ptr(), ro.data_ptr(), aux.data_ptr() if aux_mode else None, aux_mode, _stream())
    yr, rr = torch.empty_like(y), torch.empty_like(rho)
    auxr = torch.empty_like(aux)
    _lib.call("engpt_carried_residual_gauge", y.data_ptr(), rho.data_ptr(), branch.data_ptr(), _lib.BF16, *args,
              yr.data_ptr(), rr.data_ptr(), auxr.data_ptr() if aux_mode else None, aux_mode, _stream())
    torch.cuda.synchronize()
    gauged = (r0 > max_radius).sum().item()
    assert 0 < gauged < rows                        # both gauge branches are exercised
    # the two GEMMs may round a branch element to neighbouring bf16 values: compare at bf16 resolution
    assert ((yo - yr).abs().max() / yr.abs().max()).item() < 1e-2
    assert ((ro - rr).abs() / rr).max().item() < 1e-2
    assert ((yo / ro[:, None]) - (yr / rr[:, None])).abs().max().item() < 2e-2
    if aux_mode:
        assert ((aux.float() - auxr.float()).abs().max() / auxr.float().abs().max()).item() < 2e-2


def test_gemm_carried_residual_in_place_is_exact(cuda):
    """y_out = y and rho_out = rho (how the forward calls it) give bit-identical results to separate outputs."""
    rows, d, K = 777, 1024, 1024
    a, w, y, rho, alpha = _residual_case(cuda, rows, d, K, 5)
    args = (alpha.data_ptr(), 1.0, 1, 1e-6, 1e-6, 4.0, rows, d)
    yo, ro = torch.empty_like(y), torch.empty_like(rho)
    aux1 = torch.empty(rows, d, device=cuda, dtype=torch.bfloat16)
    aux2 = torch.empty_like(aux1)
    _lib.call("engpt_gemm_carried_residual", a.data_ptr(), K, w.data_ptr(), K, K, y.data_ptr(), rho.data_ptr(), *args,
              yo.data_ptr(), ro.data_ptr(), aux1.data_ptr(), _lib.AUX_BF16_H, _stream())
    yi, ri = y.clone(), rho.clone()
    _lib.call("engpt_gemm_carried_residual", a.data_ptr(), K, w.data_ptr(), K, K, yi.data_ptr(), ri.data_ptr(),
              *args, yi.data_ptr(), ri.data_ptr(), aux2.data_ptr(), _lib.AUX_BF16_H, _stream())
    torch.cuda.synchronize()
    assert torch.equal(yo, yi) and torch.equal(ro, ri) and torch.equal(aux1, aux2)


def test_gemm_carried_residual_rejects_unsupported(cuda):
    """d = 1280 would need a cluster of 5 CTAs: refused with ENGPT_ERR_UNSUPPORTED before any device work."""
    a = torch.zeros(128, 256, device=cuda, dtype=torch.bfloat16)
    w = torch.zeros(1280, 256, device=cuda, dtype=torch.bfloat16)
    y = torch.zeros(128, 1280, device=cuda)
    rho = torch.ones(128, device=cuda)
    alpha = torch.zeros(1280, device=cuda)
    with pytest.raises(_lib.EngptError) as ei:
        _lib.call("engpt_gemm_carried_residual", a.data_ptr(), 256, w.data_ptr(), 256, 256, y.data_ptr(),
                  rho.data_ptr(), alpha.data_ptr(), 1.0, 1, 1e-6, 1e-6, 0.0, 128, 1280, y.data_ptr(), rho.data_ptr(),
                  None, 0, _stream())
    assert ei.value.code == 6   # ENGPT_ERR_UNSUPPORTED


@pytest.mark.parametrize("rows,d,vocab,ld", [(300, 256, 1000, 1024), (256, 1024, 50257, 50304), (129, 512, 300, 304)])
def test_logits_cross_entropy_matches_unfused_path(cuda, rows, d, vocab, ld):
    """Head GEMM with the log-sum-exp in its epilogue + the merge kernel vs cuBLAS logits + engpt_cross_entropy and
    F.cross_entropy on the same bf16 logits (engpt/models.py:328-333), including ignore_index rows and a vocab that
    is not a multiple of the 256-column tile."""
    g = torch.Generator().manual_seed(vocab)
    x = (torch.randn(rows, d, generator=g) * 2.0).to(cuda, torch.bfloat16)
    w = (torch.randn(vocab, d, generator=g) / d ** 0.5).to(cuda, torch.bfloat16)
    tgt = torch.randint(0, vocab, (rows,), generator=g)
    tgt[::7] = -100
    tgt = tgt.to(cuda)
    tiles = -(-vocab // 256)
    logits = torch.full((rows, ld), float("nan"), device=cuda, dtype=torch.bfloat16)
    part = torch.empty(tiles * rows * 2, device=cuda)
    row_loss = torch.empty(rows, device=cuda)
    loss = torch.empty((), device=cuda)
    _lib.call("engpt_logits_cross_entropy", x.data_ptr(), w.data_ptr(), rows, d, vocab, logits.data_ptr(), ld,
              tgt.data_ptr(), part.data_ptr(), row_loss.data_ptr(), loss.data_ptr(), _stream())
    ref_logits = torch.mm(x, w.t())
    got = logits[:, :vocab].float()
    assert ((got - ref_logits.float()).abs().max() / ref_logits.float().abs().max()).item() < 1e-2
    # the loss of the fused path on its own logits equals F.cross_entropy of those logits
    ref = torch.nn.functional.cross_entropy(got, tgt, ignore_index=-100)
    assert abs(loss.item() - ref.item()) < 1e-3, (loss.item(), ref.item())
    valid = tgt != -100
    rl_ref = torch.nn.functional.cross_entropy(got, tgt.clamp(min=0), reduction="none")
    assert (row_loss[valid] - rl_ref[valid]).abs().max().item() < 2e-3
    assert (row_loss[~valid] == 0).all()
    # and the unfused production path (cuBLAS logits, then the cross-entropy kernel)
    rl2 = torch.empty_like(row_loss)
    loss2 = torch.empty((), device=cuda)
    _lib.call("engpt_cross_entropy", ref_logits.data_ptr(), _lib.BF16, rows, vocab, vocab, tgt.data_ptr(),
              rl2.data_ptr(), loss2.data_ptr(), _stream())
    assert abs(loss.item() - loss2.item()) < 1e-2


def test_torch_ops_match_python_ops(cuda):
    """torch.ops.engpt_b200.* (the registered operators) give the Python ops' results bit for bit."""
    rng = np.random.default_rng(3)
    B, T, H, Dh = 2, 100, 4, 64
    qkv = t(rng.standard_normal((B, T, 3, H, Dh)), cuda, torch.bfloat16)
    rho = t(rng.uniform(0.5, 50.0, (B, T)), cuda)
    cos, sin = K.rotary_frequencies(T, Dh, device=cuda, dtype=torch.float32, theta=10000.0)
    sc = t(rng.uniform(0.9, 1.1, (H, Dh)), cuda)
    a = K.qkv_postprocess_from_carried(qkv, rho, cos, sin, sc, 1e-6)
    b = torch.ops.engpt_b200.qkv_postprocess_from_carried(qkv, rho, cos, sin, sc, 1e-6)
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    o1 = K.causal_sdpa(*a, scale=8.0, dropout_p=0.0)
    o2 = torch.ops.engpt_b200.causal_sdpa(*b, scale=8.0, dropout_p=0.0)
    assert torch.equal(o1, o2)
    y = t(rng.standard_normal((B, T, 256)), cuda)
    br = t(rng.standard_normal((B, T, 256)), cuda, torch.bfloat16)
    al = t(rng.uniform(0, 0.1, 256), cuda)
    r1 = K.carried_residual_gauge(y, rho, br, al, 1e-6, 1e-6, 1024.0)
    r2 = torch.ops.engpt_b200.carried_residual_gauge(y, rho, br, al, 1e-6, 1e-6, 1024.0)
    assert torch.equal(r1[0], r2[0]) and torch.equal(r1[1], r2[1])


def test_carried_up_gate_swiglu_op_fused_under_autocast(cuda):
    """The op-level MLP helper (engpt/kernels.py:182-206) under bf16 autocast runs the fused up/gate + SwiGLU
    GEMM: result against an fp32 restatement of the reference formula on the same bf16 operands, and the
    reference's output dtype (fp32)."""
    g = torch.Generator().manual_seed(9)
    B, T, d, W = 2, 96, 256, 1024
    y = (torch.randn(B, T, d, generator=g) * 3).to(cuda)
    rho = (torch.rand(B, T, generator=g) * 5 + 0.5).to(cuda)
    w = (torch.randn(2 * W, d, generator=g) / 16).to(cuda)
    su = (torch.rand(W, generator=g) + 0.5).to(cuda)
    sg = (torch.rand(W, generator=g) + 0.5).to(cuda)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = K.carried_up_gate_swiglu(y, rho, w, su, sg, sqrt_d=16.0, scale_u_by_sqrt_d=True)
    assert out.dtype == torch.float32 and out.shape == (B, T, W)
    x = (y / rho.unsqueeze(-1)).to(torch.bfloat16).float()
    ug = x @ w.to(torch.bfloat16).float().t()
    u, gate = ug[..., :W] * su * 16.0, ug[..., W:] * sg * 16.0
    ref = u * torch.nn.functional.silu(gate)
    assert ((out - ref).abs().max() / ref.abs().max()).item() < 1e-2
