"""``engpt.kernels``-compatible ops backed by the sm_100a kernels of ``libengpt_b200``.

Each function keeps the name, argument meaning and return shapes of the
reference op it replaces (cited per function, paths inside the
Pi-Willie/enGPT project) and launches CUDA kernels through the C ABI on the
current torch stream.  There is no CPU or library fallback: non-CUDA inputs,
float64, and autograd-tracked inputs raise.

Ownership differs from the reference in one place: the reference's no-grad
``qkv_postprocess_from_carried`` returns views into ``qkv`` after mutating it;
here ``qkv`` is read-only and fresh tensors are returned (callers in the
reference never reuse ``qkv``).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
from torch import Tensor

from . import _lib

__all__ = [
    "normalize_rows_",
    "normalize_columns_",
    "project_row_grad_",
    "project_column_grad_",
    "qkv_postprocess_from_carried",
    "causal_sdpa",
    "ngpt_attention_scale",
    "gpt_attention_scale",
    "carried_residual_gauge",
    "carried_residual",
    "rotary_frequencies",
    "carried_up_gate_swiglu",
    "scaled_logits_from_carried",
    "attention_strides",
]


def _require_cuda(*ts: Optional[Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("engpt_b200 ops run on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("engpt_b200 ops: all tensors must be on the same device")
    return dev


def _forward_only(*ts: Optional[Tensor]) -> None:
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts):
        raise NotImplementedError("engpt_b200 kernels are forward-only; call under torch.no_grad()")


def _f32c(t: Tensor) -> Tensor:
    return t.to(torch.float32).contiguous()


def ngpt_attention_scale(head_dim: int) -> float:
    """``sqrt(head_dim)`` -- engpt/kernels.py:434-435."""
    return math.sqrt(float(head_dim))


def gpt_attention_scale(head_dim: int) -> float:
    """``1/sqrt(head_dim)`` -- engpt/kernels.py:438-439."""
    return 1.0 / math.sqrt(float(head_dim))


def rotary_frequencies(seq_len: int, head_dim: int, *, device: torch.device, dtype: torch.dtype,
                       theta: float) -> Tuple[Tensor, Tensor]:
    """cos/sin tables ``[T, rd/2]`` -- engpt/kernels.py:355-374 (computed in fp32, cast to ``dtype``)."""
    device = torch.device(device)
    rd = head_dim - (head_dim % 2)
    if rd == 0:
        empty = torch.empty(seq_len, 0, device=device, dtype=dtype)
        return empty, empty
    if device.type != "cuda":
        raise RuntimeError("engpt_b200 ops run on CUDA tensors only (no CPU fallback)")
    cos = torch.empty(seq_len, rd // 2, device=device, dtype=torch.float32)
    sin = torch.empty_like(cos)
    with torch.cuda.device(device):
        _lib.call("engpt_rotary_tables", seq_len, head_dim, float(theta), cos.data_ptr(), sin.data_ptr(),
                  _lib.stream_handle(device))
    if dtype != torch.float32:
        return cos.to(dtype), sin.to(dtype)
    return cos, sin


def qkv_postprocess_into(qkv: Tensor, rho: Tensor, cos: Tensor, sin: Tensor, qk_scale: Tensor, qk_mult: float,
                         norm_eps: float, q: Tensor, k: Tensor, v: Tensor, head_major: bool) -> None:
    """Launch the fused epilogue into caller-owned ``q, k, v`` (no checks beyond the C ABI's)."""
    bsz, seq_len, _, n_head, head_dim = qkv.shape
    _lib.call("engpt_qkv_postprocess", qkv.data_ptr(), _lib.dtype_code(qkv.dtype), rho.data_ptr(),
              cos.data_ptr() if cos.numel() else None, sin.data_ptr() if sin.numel() else None, cos.shape[-1],
              qk_scale.data_ptr(), float(qk_mult), float(norm_eps), bsz, seq_len, n_head, head_dim,
              q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.QKV_BHTD if head_major else _lib.QKV_BTHD,
              _lib.stream_handle(qkv.device))


def qkv_postprocess_from_carried(qkv: Tensor, rho: Tensor, cos: Tensor, sin: Tensor, qk_scale: Tensor,
                                 norm_eps: float) -> Tuple[Tensor, Tensor, Tensor]:
    """Raw ``[B, T, 3, H, Dh]`` projection of carried ``Y`` -> nGPT attention inputs.

    engpt/kernels.py:139-179: q/k are L2-normalised per head (norm guarded by
    ``rho * eps``), rotated with interleaved RoPE and scaled by ``qk_scale``;
    v is divided by ``rho``.  Returns ``[B, T, H, Dh]`` tensors in ``qkv.dtype``.
    """
    _require_cuda(qkv, rho, cos, sin, qk_scale)
    _forward_only(qkv, rho, cos, sin, qk_scale)
    if qkv.dim() != 5 or qkv.shape[2] != 3:
        raise ValueError("qkv must have shape [B, T, 3, H, Dh]")
    bsz, seq_len, _, n_head, head_dim = qkv.shape
    if tuple(rho.shape) != (bsz, seq_len):
        raise ValueError("rho must have shape [batch, sequence]")
    if tuple(qk_scale.shape) != (n_head, head_dim):
        raise ValueError("qk_scale must have shape [n_head, head_dim]")
    half = (head_dim - head_dim % 2) // 2
    if cos.shape[-1] != half or cos.shape[0] < seq_len or sin.shape != cos.shape:
        raise ValueError("cos/sin must have shape [T, head_dim // 2]")
    qkv = qkv.contiguous()
    out = [torch.empty(bsz, seq_len, n_head, head_dim, device=qkv.device, dtype=qkv.dtype) for _ in range(3)]
    with torch.cuda.device(qkv.device):
        qkv_postprocess_into(qkv, _f32c(rho), _f32c(cos[:seq_len]), _f32c(sin[:seq_len]), _f32c(qk_scale), 1.0,
                             norm_eps, out[0], out[1], out[2], head_major=False)
    return out[0], out[1], out[2]


def attention_strides(q: Tensor, k: Tensor, v: Tensor, o: Tensor, head_major: bool) -> torch.Tensor:
    """Element strides (batch, token, head) of four ``[B,T,H,D]`` (or ``[B,H,T,D]``) tensors."""
    vals = []
    for t in (q, k, v, o):
        if t.stride(-1) != 1:
            raise ValueError("attention inputs need a contiguous head_dim axis")
        s = t.stride()
        vals += [s[0], s[2], s[1]] if head_major else [s[0], s[1], s[2]]
    return torch.tensor(vals, dtype=torch.int64)


def causal_attention_into(q: Tensor, k: Tensor, v: Tensor, o: Tensor, scale: float, strides: torch.Tensor,
                          bsz: int, seq_len: int, n_head: int, head_dim: int, impl: int = _lib.ATTN_AUTO) -> None:
    _lib.call("engpt_causal_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
              _lib.dtype_code(q.dtype), bsz, seq_len, n_head, head_dim, float(scale), strides.data_ptr(), impl,
              _lib.stream_handle(q.device))


def causal_sdpa(q: Tensor, k: Tensor, v: Tensor, *, scale: float, dropout_p: float, impl: str = "auto") -> Tensor:
    """Causal softmax attention on ``[B, T, H, D]`` inputs, returning ``[B, T, H, D]``.

    engpt/kernels.py:417-431 (``softmax(scale * q k^T + causal mask) v``).
    bf16 inputs with head_dim 64 or 128 run on the tcgen05 kernel; fp32 and
    other head dims run on the CUDA-core kernel.  ``impl`` ("auto",
    "tcgen05", "simt") forces a kernel.
    """
    _require_cuda(q, k, v)
    _forward_only(q, k, v)
    if dropout_p:
        raise NotImplementedError("engpt_b200 attention is inference-only (dropout_p must be 0)")
    if q.dim() != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must share shape [B, T, H, D]")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, v must share a dtype")
    bsz, seq_len, n_head, head_dim = q.shape
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (q, k, v))
    o = torch.empty(bsz, seq_len, n_head, head_dim, device=q.device, dtype=q.dtype)
    strides = attention_strides(q, k, v, o, head_major=False)
    code = {"auto": _lib.ATTN_AUTO, "tcgen05": _lib.ATTN_TCGEN05, "simt": _lib.ATTN_SIMT,
            "tcgen05_1tile": _lib.ATTN_TCGEN05_1TILE}[impl]
    with torch.cuda.device(q.device):
        causal_attention_into(q, k, v, o, scale, strides, bsz, seq_len, n_head, head_dim, code)
    return o


def carried_residual_into(y: Tensor, rho: Tensor, branch: Tensor, alpha: Tensor, alpha_mult: float,
                          alpha_abs: bool, branch_eps: float, residual_eps: float, max_radius: float,
                          y_out: Tensor, rho_out: Tensor, aux: Optional[Tensor], aux_mode: int) -> None:
    rows = rho.numel()
    d = y.shape[-1]
    _lib.call("engpt_carried_residual_gauge", y.data_ptr(), rho.data_ptr(), branch.data_ptr(),
              _lib.dtype_code(branch.dtype), alpha.data_ptr(), float(alpha_mult), 1 if alpha_abs else 0,
              float(branch_eps), float(residual_eps), float(max_radius), rows, d, y_out.data_ptr(),
              rho_out.data_ptr(), None if aux is None else aux.data_ptr(), aux_mode, _lib.stream_handle(y.device))


def carried_residual_gauge(y: Tensor, rho: Tensor, branch: Tensor, alpha: Tensor, branch_eps: float,
                           residual_eps: float, max_radius: float) -> Tuple[Tensor, Tensor]:
    """Carried nGPT residual with the exact gauge rescale, in one pass.

    engpt/kernels.py:277-324.  ``y`` ``[..., d]`` and ``rho`` ``[...]`` are
    carried in fp32 (as in the reference's autocast flow); ``branch`` may be
    bf16 or fp32; ``alpha`` is ``[d]`` (leading singleton dims allowed).
    """
    _require_cuda(y, rho, branch, alpha)
    _forward_only(y, rho, branch, alpha)
    if branch.shape != y.shape or tuple(rho.shape) != tuple(y.shape[:-1]):
        raise ValueError("y/branch must be [..., d] and rho [...]")
    d = y.shape[-1]
    if alpha.numel() != d:
        raise ValueError("alpha must have d elements")
    out_dtype = torch.promote_types(y.dtype, branch.dtype)
    yc = _f32c(y)
    bc = branch.contiguous() if branch.dtype in (torch.bfloat16, torch.float32) else branch.float().contiguous()
    y_out = torch.empty(y.shape, device=y.device, dtype=torch.float32)
    rho_out = torch.empty(rho.shape, device=y.device, dtype=torch.float32)
    with torch.cuda.device(y.device):
        carried_residual_into(yc, _f32c(rho), bc, _f32c(alpha.reshape(-1)), 1.0, False, branch_eps, residual_eps,
                              max_radius, y_out, rho_out, None, _lib.AUX_NONE)
    if out_dtype != torch.float32:
        return y_out.to(out_dtype), rho_out.to(out_dtype)
    return y_out, rho_out


def carried_residual(y: Tensor, rho: Tensor, branch: Tensor, alpha: Tensor, branch_eps: float,
                     residual_eps: float) -> Tuple[Tensor, Tensor]:
    """engpt/kernels.py:232-274: the residual without the gauge (``max_radius <= 0``)."""
    return carried_residual_gauge(y, rho, branch, alpha, branch_eps, residual_eps, 0.0)


def swiglu_into(ug: Tensor, s_u: Tensor, s_gate: Tensor, u_mult: float, gate_mult: float, out: Tensor) -> None:
    width = out.shape[-1]
    rows = out.numel() // width
    _lib.call("engpt_swiglu", ug.data_ptr(), _lib.dtype_code(ug.dtype), s_u.data_ptr(), s_gate.data_ptr(),
              float(u_mult), float(gate_mult), rows, width, out.data_ptr(), _lib.dtype_code(out.dtype),
              _lib.stream_handle(ug.device))


def carried_up_gate_swiglu(y: Tensor, rho: Tensor, weight: Tensor, s_u: Tensor, s_gate: Tensor, *, sqrt_d: float,
                           scale_u_by_sqrt_d: bool) -> Tensor:
    """MLP up/gate projection of ``Y/rho`` + SwiGLU -- engpt/kernels.py:182-206.

    Under bf16 autocast (the reference's GPU flow) with a width that is a
    multiple of 128: the tcgen05 GEMM with SwiGLU in its epilogue
    (``engpt_up_gate_swiglu``), so the ``[.., 2W]`` projection is never
    written; otherwise a cuBLAS GEMM (through torch, honouring autocast) and
    the SwiGLU kernel.  The result has the reference's dtype (bf16 GEMM output
    times fp32 scales: fp32).
    """
    _require_cuda(y, rho, weight, s_u, s_gate)
    _forward_only(y, rho, weight, s_u, s_gate)
    mlp_in = y / rho.unsqueeze(-1)
    d = mlp_in.shape[-1]
    width = weight.shape[0] // 2
    if (torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
            and width % 128 == 0 and d % 8 == 0 and weight.shape[1] == d):
        x = mlp_in.reshape(-1, d).to(torch.bfloat16).contiguous()
        w = weight.to(torch.bfloat16).contiguous()
        hidden = torch.empty(x.shape[0], width, device=x.device, dtype=torch.bfloat16)
        su, sg = _f32c(s_u), _f32c(s_gate)
        with torch.cuda.device(y.device):
            _lib.call("engpt_up_gate_swiglu", x.data_ptr(), w.data_ptr(), su.data_ptr(), sg.data_ptr(),
                      float(sqrt_d if scale_u_by_sqrt_d else 1.0), float(sqrt_d), x.shape[0], d, width,
                      hidden.data_ptr(), _lib.stream_handle(y.device))
        out_dtype = torch.promote_types(torch.bfloat16, s_u.dtype)
        return hidden.view(*mlp_in.shape[:-1], width).to(out_dtype)
    ug = torch.nn.functional.linear(mlp_in, weight).contiguous()
    width = ug.shape[-1] // 2
    out = torch.empty(*ug.shape[:-1], width, device=ug.device, dtype=torch.promote_types(ug.dtype, s_u.dtype))
    with torch.cuda.device(y.device):
        swiglu_into(ug, _f32c(s_u), _f32c(s_gate), sqrt_d if scale_u_by_sqrt_d else 1.0, sqrt_d, out)
    return out


def scaled_logits_from_carried(y: Tensor, rho: Tensor, output_emb: Tensor, logit_scale: Tensor) -> Tensor:
    """``<Y, E_out[v]> s_z[v] / rho`` -- engpt/kernels.py:209-229 (cuBLAS GEMM on row-scaled weights)."""
    _require_cuda(y, rho, output_emb, logit_scale)
    _forward_only(y, rho, output_emb, logit_scale)
    h = y / rho.unsqueeze(-1)
    w = torch.empty(output_emb.shape, device=y.device,
                    dtype=torch.bfloat16 if torch.is_autocast_enabled("cuda") else torch.float32)
    emb32, scale32 = _f32c(output_emb), _f32c(logit_scale)
    with torch.cuda.device(y.device):
        _lib.call("engpt_scale_rows_cast", emb32.data_ptr(), scale32.data_ptr(), 1.0, output_emb.shape[0],
                  output_emb.shape[1], w.data_ptr(), _lib.dtype_code(w.dtype), _lib.stream_handle(y.device))
    return torch.nn.functional.linear(h.to(w.dtype), w)


# ------------------------------------------------------------ optimizer-side sphere operations
def _sphere_matrix(x: Tensor, what: str) -> None:
    if not x.is_cuda:
        raise RuntimeError("engpt_b200 ops run on CUDA tensors only (no CPU fallback)")
    if x.ndim != 2 or not x.is_contiguous():
        raise ValueError(f"{what}: needs a contiguous 2-D matrix, got shape {tuple(x.shape)}")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise NotImplementedError(f"{what}: float32 and bfloat16 only, got {x.dtype}")


@torch.no_grad()
def normalize_rows_(x: Tensor, eps: float = 1e-12) -> Tensor:
    """In place: every row to unit L2 norm, ``x[r] /= max(|x[r]|, eps)`` -- engpt/kernels.py:98-105."""
    _sphere_matrix(x, "normalize_rows_")
    with torch.cuda.device(x.device):
        _lib.call("engpt_normalize_rows", x.data_ptr(), _lib.dtype_code(x.dtype), x.shape[0], x.shape[1],
                  float(eps), _lib.stream_handle(x.device))
    return x


def _column_scratch(x: Tensor) -> Tensor:
    n = int(_lib.load().engpt_column_scratch_floats(x.shape[0], x.shape[1]))
    return torch.empty(max(n, 1), device=x.device, dtype=torch.float32)


@torch.no_grad()
def normalize_columns_(x: Tensor, eps: float = 1e-12) -> Tensor:
    """In place: every column to unit L2 norm, ``x[:, c] /= max(|x[:, c]|, eps)`` -- engpt/kernels.py:108-116."""
    _sphere_matrix(x, "normalize_columns_")
    scratch = _column_scratch(x)
    with torch.cuda.device(x.device):
        _lib.call("engpt_normalize_columns", x.data_ptr(), _lib.dtype_code(x.dtype), x.shape[0], x.shape[1],
                  float(eps), scratch.data_ptr(), _lib.stream_handle(x.device))
    return x


def _check_pair(weight: Tensor, grad: Tensor, what: str) -> None:
    _sphere_matrix(weight, what)
    _sphere_matrix(grad, what)
    if weight.shape != grad.shape or weight.dtype != grad.dtype or weight.device != grad.device:
        raise ValueError(f"{what}: weight and grad must share shape, dtype and device")


@torch.no_grad()
def project_row_grad_(weight: Tensor, grad: Tensor) -> None:
    """In place: ``grad[r] -= (grad[r] . weight[r]) weight[r]`` (tangent space of unit rows) --
    engpt/kernels.py:119-125."""
    _check_pair(weight, grad, "project_row_grad_")
    with torch.cuda.device(grad.device):
        _lib.call("engpt_project_row_grad", weight.data_ptr(), grad.data_ptr(), _lib.dtype_code(grad.dtype),
                  grad.shape[0], grad.shape[1], _lib.stream_handle(grad.device))


@torch.no_grad()
def project_column_grad_(weight: Tensor, grad: Tensor) -> None:
    """In place: ``grad[:, c] -= (grad[:, c] . weight[:, c]) weight[:, c]`` (tangent space of unit columns) --
    engpt/kernels.py:128-136."""
    _check_pair(weight, grad, "project_column_grad_")
    scratch = _column_scratch(grad)
    with torch.cuda.device(grad.device):
        _lib.call("engpt_project_column_grad", weight.data_ptr(), grad.data_ptr(), _lib.dtype_code(grad.dtype),
                  grad.shape[0], grad.shape[1], scratch.data_ptr(), _lib.stream_handle(grad.device))
