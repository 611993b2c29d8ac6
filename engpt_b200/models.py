"""``EfficientNGPT`` with the B200 forward engine.

The module tree, parameter names, shapes, registration order and
initialisation follow engpt/models.py:111-391, so ``state_dict`` keys match
the reference and ``torch.manual_seed(s); EfficientNGPT(cfg)`` produces the
reference's weights bit-for-bit (the init runs on the CPU with the same
random draws).  ``forward`` / ``forward_carried`` run the carried-radius
forward (engpt/models.py:263-292) on the GPU; under bf16 autocast:

  per block (engpt/models.py:140-182)
    q, k, v  = post-process(Y_bf16 @ W_qkv^T)            engpt_qkv_projection (tcgen05 GEMM, post-process in
                                                         the epilogue; head_dim 64 / 128)
    attn     = causal attention  -> [B,T,H,Dh]           engpt_ngpt_attention (tcgen05, softmax offset from the
                                                         s_qk score bound)
    branch   = attn @ W_o^T                              cuBLAS
    Y, rho   = carried residual + gauge, emits bf16 Y/rho engpt_carried_residual_gauge
    hidden   = SwiGLU((Y/rho)_bf16 @ W_ug^T)             engpt_up_gate_swiglu (tcgen05 GEMM, SwiGLU epilogue)
    branch   = hidden @ W_down^T                         cuBLAS
    Y, rho   = carried residual + gauge, emits bf16 Y    engpt_carried_residual_gauge
  logits, loss = head GEMM with the log-sum-exp          engpt_logits_cross_entropy (tcgen05 GEMM + merge;
                 per 256-column tile in its epilogue     without targets: cuBLAS logits)

Outside autocast (fp32 mode) the projections are fp32 cuBLAS GEMMs, the
attention the fp32 CUDA-core kernel and SwiGLU / cross-entropy their own
kernels.  Precision follows the reference's: under autocast the carried
state ``Y, rho`` stays fp32, GEMM operands and outputs, Q/K/V, attention
output and logits are bf16, and the loss is fp32.  All activations live in a
per-shape workspace that is reused across calls; returned logits and loss
are fresh.  ``set_head_split`` runs the forward as one rank of a group that
shares each sequence's heads and MLP units (``engpt_b200.head_split``).
"""

from __future__ import annotations

import ctypes
import math
from typing import Callable, Dict, Optional, Tuple

import torch
from torch import Tensor, nn

from . import _lib
from . import kernels as K
from .config import ModelConfig
from .head_split import HeadSplit


def _ngpt_base_scale(cfg: ModelConfig) -> float:
    return 1.0 / math.sqrt(float(cfg.n_embd))


@torch.no_grad()
def _normalize_rows_(x: Tensor, eps: float) -> None:
    # parameter retraction (engpt/kernels.py:98-105): the CUDA kernel for CUDA parameters; on the CPU (the
    # seeded init, which must reproduce the reference's weights bit for bit) the reference's PyTorch expression
    if x.is_cuda:
        K.normalize_rows_(x, eps)
    else:
        x.div_(torch.linalg.vector_norm(x, ord=2, dim=-1, keepdim=True).clamp_min(eps))


@torch.no_grad()
def _normalize_columns_(x: Tensor, eps: float) -> None:
    # engpt/kernels.py:108-116, as _normalize_rows_
    if x.is_cuda:
        K.normalize_columns_(x, eps)
    else:
        x.div_(torch.linalg.vector_norm(x, ord=2, dim=0, keepdim=True).clamp_min(eps))


class EfficientNGPTBlock(nn.Module):
    """One carried-radius nGPT block; parameters as engpt/models.py:111-126."""

    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.qkv = nn.Linear(cfg.n_embd, 3 * cfg.n_embd, bias=False)
        self.out_proj = nn.Linear(cfg.n_embd, cfg.n_embd, bias=False)
        self.up_gate = nn.Linear(cfg.n_embd, 2 * cfg.mlp_width, bias=False)
        self.down_proj = nn.Linear(cfg.mlp_width, cfg.n_embd, bias=False)
        base_scale = _ngpt_base_scale(cfg)
        self.alpha_init_value = cfg.alpha_init
        self.scalar_init_scaling = base_scale
        self.alpha_attn_raw = nn.Parameter(torch.full((cfg.n_embd,), base_scale))
        self.alpha_mlp_raw = nn.Parameter(torch.full((cfg.n_embd,), base_scale))
        self.s_qk = nn.Parameter(torch.full((cfg.n_head, cfg.head_dim), base_scale))
        self.s_u = nn.Parameter(torch.ones(cfg.mlp_width))
        self.s_gate = nn.Parameter(torch.ones(cfg.mlp_width))

    # effective scalars (engpt/models.py:128-138), as multipliers on the raw parameters
    @property
    def alpha_mult(self) -> float:
        return self.alpha_init_value / self.scalar_init_scaling

    @property
    def qk_mult(self) -> float:
        return 1.0 / self.scalar_init_scaling

    @property
    def alpha_attn(self) -> Tensor:
        return self.alpha_attn_raw.abs() * self.alpha_mult

    @property
    def alpha_mlp(self) -> Tensor:
        return self.alpha_mlp_raw.abs() * self.alpha_mult

    @property
    def qk_scale(self) -> Tensor:
        return self.s_qk * self.qk_mult

    def forward(self, y: Tensor, rho: Tensor, cos: Tensor, sin: Tensor) -> Tuple[Tensor, Tensor]:
        """engpt/models.py:140-182 through the engpt_b200 ops (standalone block call)."""
        cfg = self.cfg
        bsz, seq_len, _ = y.shape
        qkv = self.qkv(y).view(bsz, seq_len, 3, cfg.n_head, cfg.head_dim)
        q, k, v = K.qkv_postprocess_from_carried(qkv, rho, cos, sin, self.qk_scale, cfg.norm_eps)
        attn = K.causal_sdpa(q, k, v, scale=K.ngpt_attention_scale(cfg.head_dim), dropout_p=0.0)
        branch = self.out_proj(attn.reshape(bsz, seq_len, -1))
        y, rho = K.carried_residual_gauge(y, rho, branch, self.alpha_attn, cfg.norm_eps, cfg.norm_eps,
                                          cfg.carried_gauge_max)
        hidden = K.carried_up_gate_swiglu(y, rho, self.up_gate.weight, self.s_u, self.s_gate,
                                          sqrt_d=math.sqrt(float(cfg.n_embd)),
                                          scale_u_by_sqrt_d=cfg.scale_mlp_u_by_sqrt_d)
        branch = self.down_proj(hidden)
        return K.carried_residual_gauge(y, rho, branch, self.alpha_mlp, cfg.norm_eps, cfg.norm_eps,
                                        cfg.carried_gauge_max)

    @torch.no_grad()
    def project_parameters_(self, eps: float = 1e-12) -> None:
        """engpt/models.py:223-230."""
        _normalize_rows_(self.qkv.weight, eps)
        _normalize_columns_(self.out_proj.weight, eps)
        _normalize_rows_(self.up_gate.weight, eps)
        _normalize_columns_(self.down_proj.weight, eps)


class _Workspace:
    """Activation buffers for one (batch, seq_len, precision) shape on one device."""

    def __init__(self, cfg: ModelConfig, bsz: int, seq_len: int, device: torch.device, bf16: bool,
                 fuse_mlp: bool = True, split: Optional[HeadSplit] = None):
        d, Dh, W_full = cfg.n_embd, cfg.head_dim, cfg.mlp_width
        # with a head split this rank's heads and MLP units; the carried state stays full width
        H = cfg.n_head // (split.size if split else 1)
        W = W_full // (split.size if split else 1)
        dl = H * Dh                           # width of this rank's heads
        n = bsz * seq_len
        act = torch.bfloat16 if bf16 else torch.float32
        e = lambda *shape, dtype=act: torch.empty(*shape, device=device, dtype=dtype)  # noqa: E731
        self.key = (bsz, seq_len, bf16, device, fuse_mlp, split.key() if split else None)
        self.H, self.W, self.dl = H, W, dl
        self.bsz, self.seq_len, self.n = bsz, seq_len, n
        self.act = act
        self.y = e(n, d, dtype=torch.float32)
        self.rho = e(n, dtype=torch.float32)
        self.x = e(n, d)                      # GEMM operand: Y (QKV) or Y/rho (up/gate, head)
        # raw projection [B, T, 3, H, Dh]; the epilogue turns it into q, k, v in place
        self.qkv = e(n, 3 * dl)
        qkv5 = self.qkv.view(bsz, seq_len, 3, H, Dh)
        self.q, self.k, self.v = qkv5[:, :, 0], qkv5[:, :, 1], qkv5[:, :, 2]   # [B, T, H, Dh] views
        self.attn = e(n, dl)                  # [B, T, H, Dh]
        self.branch = e(n, d)
        # bf16 mode fuses SwiGLU into the up/gate GEMM (no [n, 2W] buffer); fp32 mode runs cuBLAS + the
        # SwiGLU kernel
        self.ug = None if (bf16 and fuse_mlp and W % 128 == 0 and d % 8 == 0) else e(n, 2 * W)
        self.hidden = e(n, W)
        self.row_loss = e(n, dtype=torch.float32)
        self.cos = e(seq_len, Dh // 2, dtype=torch.float32)
        self.sin = e(seq_len, Dh // 2, dtype=torch.float32)
        self.attn_strides = K.attention_strides(self.q, self.k, self.v, self.attn.view(bsz, seq_len, H, Dh),
                                                head_major=False)
        # bf16 weight copies (re-cast from the fp32 parameters on every forward); with a head split the QKV
        # and up/gate copies hold this rank's rows only, out_proj and down_proj are used through column views
        if bf16:
            self.w = [dict(qkv=e(3 * dl, d), out=e(d, d), ug=e(2 * W, d), down=e(d, W_full))
                      for _ in range(cfg.n_layer)]
        else:
            self.w = None
        # output-head weight with the vocab rounded up to a multiple of 64 rows (pad rows stay zero):
        # an odd vocab (50257) would give the logits GEMM an unaligned leading dimension, which
        # sends cuBLAS to a ~10x slower kernel
        self.vocab_pad = -(-cfg.vocab_size // 64) * 64
        self.w_head = torch.zeros(self.vocab_pad, d, device=device, dtype=act)
        self._lse = None
        self._lse_shape = (-(-cfg.vocab_size // 256) * n * 2,)
        self._device = device

    def lse_partials(self) -> torch.Tensor:
        """Scratch of the fused head: one (max, sum) pair per row and 256-column logits tile."""
        if self._lse is None:
            self._lse = torch.empty(self._lse_shape, device=self._device, dtype=torch.float32)
        return self._lse


class _GraphedForward:
    """One captured forward: static id / target buffers on the device, the graph, and its output buffers.

    It keeps the workspace it was captured with alive (the graph holds raw
    pointers into it), whatever the model's current workspace becomes.
    """

    def __init__(self, model: "EfficientNGPT", shape: tuple, has_targets: bool, dev: torch.device) -> None:
        self.idx = torch.zeros(shape, dtype=torch.int64, device=dev)
        self.targets = torch.zeros(shape, dtype=torch.int64, device=dev) if has_targets else None
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            model._run(idx=self.idx, targets=self.targets)   # warm-up: workspace, tensor maps, library handles
        torch.cuda.current_stream(dev).wait_stream(side)
        with torch.cuda.graph(self.graph):
            self.logits, self.loss = model._run(idx=self.idx, targets=self.targets)
        self.ws = model._ws

    def replay(self, idx: Tensor, targets: Optional[Tensor]) -> Tuple[Tensor, Optional[Tensor]]:
        self.idx.copy_(idx, non_blocking=True)
        if targets is not None:
            self.targets.copy_(targets, non_blocking=True)
        self.graph.replay()
        return self.logits, self.loss


class EfficientNGPT(nn.Module):
    """Carried-radius nGPT (engpt/models.py:233-391) with a fused B200 forward."""

    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.gradient_checkpointing = False
        self.token_emb = nn.Embedding(cfg.vocab_size, cfg.n_embd)
        self.blocks = nn.ModuleList([EfficientNGPTBlock(cfg) for _ in range(cfg.n_layer)])
        self.output_emb = nn.Parameter(torch.empty(cfg.vocab_size, cfg.n_embd))
        self.scalar_init_scaling = _ngpt_base_scale(cfg)
        self.logit_scale_init_value = cfg.logit_scale_init
        self.s_z = nn.Parameter(torch.full((cfg.vocab_size,), self.scalar_init_scaling))
        self.apply(self._init_weights)
        nn.init.normal_(self.output_emb, mean=0.0, std=0.02)
        self.project_parameters_()
        self._ws: Optional[_Workspace] = None
        self.attn_impl = _lib.ATTN_AUTO
        # bf16 mode: up/gate projection and SwiGLU in one tcgen05 GEMM (False: cuBLAS + SwiGLU kernel)
        self.fuse_mlp = True
        # bf16 mode, head_dim 64 or 128: QKV projection and its post-process in one tcgen05 GEMM (False:
        # cuBLAS + the QKV epilogue kernel in place)
        self.fuse_qkv = True
        # bf16 mode, d in {256, 512, 768, 1024}: out_proj / down_proj GEMMs with the carried residual in
        # their epilogue (engpt_gemm_carried_residual).  Off by default: at d=1024, T=2048, B=32 it measures
        # slower than cuBLAS + the carried-residual kernel (0.29 vs 0.23 ms out_proj, 0.58 vs 0.48 ms down)
        self.fuse_residual = False
        # bf16 mode with targets: output-head GEMM with the cross-entropy's log-sum-exp in its epilogue
        # (engpt_logits_cross_entropy; False: cuBLAS logits + the cross-entropy kernel)
        self.fuse_head = True
        # False: logits are a strided [B, T, V] view of a [N, V rounded up to 64] buffer (no copy);
        # True: a contiguous copy is returned
        self.contiguous_logits = False
        # optional instrumentation: called around the attention launch of every layer
        self.attn_timer: Optional[Callable[[str], None]] = None
        # this rank's share of a head-split group (set_head_split), or None for the whole model
        self.head_split: Optional[HeadSplit] = None
        # forward(idx, targets) replays one CUDA graph per input shape (captured on first use) instead of
        # launching ~10 kernels per layer from Python; see enable_cuda_graphs
        self.cuda_graphs = False
        self._graphs: Dict[tuple, "_GraphedForward"] = {}

    def _init_weights(self, module: nn.Module) -> None:
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)

    @property
    def logit_mult(self) -> float:
        return self.logit_scale_init_value / self.scalar_init_scaling

    @property
    def logit_scale(self) -> Tensor:
        return self.s_z * self.logit_mult

    @torch.no_grad()
    def project_parameters_(self, eps: float = 1e-12) -> None:
        """engpt/models.py:356-361."""
        _normalize_rows_(self.token_emb.weight, eps)
        _normalize_rows_(self.output_emb, eps)
        for block in self.blocks:
            block.project_parameters_(eps)

    def set_gradient_checkpointing(self, enabled: bool = True) -> None:
        self.gradient_checkpointing = enabled

    # ---------------------------------------------------------------- forward
    def _check_inference(self) -> None:
        if torch.is_grad_enabled() and any(p.requires_grad for p in self.parameters()):
            raise NotImplementedError(
                "engpt_b200 EfficientNGPT is a forward-only (inference) engine: call it under torch.no_grad() "
                "or after model.requires_grad_(False)")

    def forward(self, idx: Tensor, targets: Optional[Tensor] = None) -> Tuple[Tensor, Optional[Tensor]]:
        """engpt/models.py:263-268: embed, rho = 1, then the carried forward."""
        self._check_inference()
        if idx.size(1) > self.cfg.block_size:
            raise ValueError("sequence length exceeds block_size")
        if self.cuda_graphs and self.head_split is None:
            return self._graphed(idx, targets)
        return self._run(idx=idx, targets=targets)

    # ---------------------------------------------------------------- CUDA graphs
    def enable_cuda_graphs(self, enabled: bool = True) -> None:
        """Replay ``forward(idx, targets)`` from CUDA graphs, one per (batch, sequence, targets, autocast) key.

        The first call with a key runs the forward once eagerly (warm-up) and
        captures a second run; later calls copy ``idx`` / ``targets`` into the
        graph's input buffers and replay it.  The graph reads the parameters in
        place, so in-place updates (an optimizer step, ``load_state_dict``) are
        seen; parameters moved to new storage (``.to()`` of another device or
        dtype, reassigned tensors) need ``reset_cuda_graphs()``.  The returned
        ``logits`` and ``loss`` are the graph's output buffers: the next replay of
        the same key overwrites them (clone to keep them).  A head-split model
        runs eagerly (its all-reduces go through the process group).
        """
        self.cuda_graphs = enabled
        if not enabled:
            self.reset_cuda_graphs()

    def reset_cuda_graphs(self) -> None:
        self._graphs.clear()

    def _param_key(self) -> tuple:
        return (self.token_emb.weight.data_ptr(), self.output_emb.data_ptr(), self.s_z.data_ptr(),
                self.blocks[0].qkv.weight.data_ptr(), self.blocks[-1].down_proj.weight.data_ptr())

    def _graphed(self, idx: Tensor, targets: Optional[Tensor]) -> Tuple[Tensor, Optional[Tensor]]:
        dev = self.token_emb.weight.device
        if dev.type != "cuda":
            raise RuntimeError("engpt_b200 EfficientNGPT runs on CUDA only (no CPU fallback); call .cuda()")
        if targets is not None and targets.shape != idx.shape:
            raise NotImplementedError("engpt_b200 implements token targets [batch, sequence] only")
        key = (tuple(idx.shape), targets is not None, self._mode_bf16(dev), dev, self.fuse_mlp, self.fuse_qkv,
               self.fuse_residual, self.fuse_head, self.attn_impl, self.contiguous_logits, self._param_key())
        g = self._graphs.get(key)
        if g is None:
            g = _GraphedForward(self, tuple(idx.shape), targets is not None, dev)
            self._graphs[key] = g
        return g.replay(idx, targets)

    def forward_carried(self, y: Tensor, rho: Tensor,
                        targets: Optional[Tensor] = None) -> Tuple[Tensor, Optional[Tensor]]:
        """engpt/models.py:270-292 from an explicit carried state ``(y, rho)`` (any rho > 0)."""
        self._check_inference()
        if y.size(1) > self.cfg.block_size:
            raise ValueError("sequence length exceeds block_size")
        if rho.shape != y.shape[:2]:
            raise ValueError("rho must have shape [batch, sequence]")
        return self._run(y=y, rho=rho, targets=targets)

    @staticmethod
    def loss_from_logits(logits: Tensor, targets: Optional[Tensor]) -> Optional[Tensor]:
        """engpt/models.py:328-339 (token targets) on the CUDA cross-entropy kernel."""
        if targets is None:
            return None
        if targets.ndim != logits.ndim - 1:
            raise NotImplementedError("engpt_b200 implements token targets [batch, sequence] only")
        v = logits.shape[-1]
        flat = logits.reshape(-1, v)
        if flat.stride(-1) != 1:
            flat = flat.contiguous()
        t = targets.reshape(-1).to(device=logits.device, dtype=torch.int64).contiguous()
        row_loss = torch.empty(flat.shape[0], device=logits.device, dtype=torch.float32)
        loss = torch.empty((), device=logits.device, dtype=torch.float32)
        with torch.cuda.device(logits.device):
            _lib.call("engpt_cross_entropy", flat.data_ptr(), _lib.dtype_code(flat.dtype), flat.shape[0], v,
                      flat.stride(0), t.data_ptr(), row_loss.data_ptr(), loss.data_ptr(),
                      _lib.stream_handle(logits.device))
        return loss

    def _workspace(self, bsz: int, seq_len: int, device: torch.device, bf16: bool) -> _Workspace:
        split = self.head_split
        key = (bsz, seq_len, bf16, device, self.fuse_mlp, split.key() if split else None)
        if self._ws is None or self._ws.key != key:
            self._ws = None
            self._ws = _Workspace(self.cfg, bsz, seq_len, device, bf16, self.fuse_mlp, split)
        return self._ws

    def set_head_split(self, split: Optional[HeadSplit]) -> None:
        """Run the forward as one rank of a head-split group (``engpt_b200.head_split``), or whole (None).

        Every rank of the group holds the full weights and calls ``forward`` on the
        same ids; each computes its heads and MLP units, and the partial branches are
        summed over the group before every carried residual, so all ranks return the
        same logits and loss.
        """
        if split is not None:
            split.validate(self.cfg.n_head, self.cfg.mlp_width)
            if split.size == 1:
                split = None
        self.head_split = split
        self._ws = None

    def release_workspace(self) -> None:
        self._ws = None

    def _mode_bf16(self, device: torch.device) -> bool:
        p = self.token_emb.weight
        if p.dtype != torch.float32:
            raise NotImplementedError(f"engpt_b200 forward runs fp32 parameters (got {p.dtype})")
        if torch.is_autocast_enabled("cuda"):
            dt = torch.get_autocast_dtype("cuda")
            if dt != torch.bfloat16:
                raise NotImplementedError(f"engpt_b200 forward supports bf16 autocast only (got {dt})")
            return True
        return False

    @torch.no_grad()
    def _run(self, idx: Optional[Tensor] = None, y: Optional[Tensor] = None, rho: Optional[Tensor] = None,
             targets: Optional[Tensor] = None,
             layer_callback: Optional[Callable[[int, Tensor, Tensor], None]] = None
             ) -> Tuple[Tensor, Optional[Tensor]]:
        cfg = self.cfg
        dev = self.token_emb.weight.device
        if dev.type != "cuda":
            raise RuntimeError("engpt_b200 EfficientNGPT runs on CUDA only (no CPU fallback); call .cuda()")
        bf16 = self._mode_bf16(dev)
        src = idx if idx is not None else y
        bsz, seq_len = src.shape[0], src.shape[1]
        n = bsz * seq_len
        d, H, Dh, W = cfg.n_embd, cfg.n_head, cfg.head_dim, cfg.mlp_width
        # head split (engpt_b200.head_split): this rank's heads [h0, h1) and MLP units [u0, u1)
        split = self.head_split
        h0, h1 = split.heads(H) if split else (0, H)
        u0, u1 = split.units(W) if split else (0, W)
        Hl, dl, Wl = h1 - h0, (h1 - h0) * Dh, u1 - u0
        ws = self._workspace(bsz, seq_len, dev, bf16)
        st = _lib.stream_handle(dev)
        act = _lib.dtype_code(ws.act)
        with torch.cuda.device(dev):
            # rotary tables (engpt/models.py:280 -> engpt/kernels.py:355-374)
            if Dh // 2 > 0:
                _lib.call("engpt_rotary_tables", seq_len, Dh, float(cfg.rope_theta), ws.cos.data_ptr(),
                          ws.sin.data_ptr(), st)
            # carried embedding (engpt/models.py:266-267)
            if idx is not None:
                ids = idx.to(device=dev, dtype=torch.int64, non_blocking=True).contiguous()
                _lib.call("engpt_embed_carried", ids.data_ptr(), self.token_emb.weight.data_ptr(), n, d,
                          cfg.vocab_size, ws.y.data_ptr(), ws.rho.data_ptr(),
                          ws.x.data_ptr() if bf16 else None, st)
            else:
                ws.y.copy_(y.reshape(n, d))
                ws.rho.copy_(rho.reshape(n))
                if bf16:
                    _lib.call("engpt_scale_rows_cast", ws.y.data_ptr(), None, 1.0, n, d, ws.x.data_ptr(),
                              _lib.BF16, st)
            if bf16:
                # autocast's per-forward bf16 copies of the linear weights, in one batched launch
                srcs, dsts, counts = [], [], []

                def add(src, src_row, dst, dst_row, nrows):   # rows [src_row, +nrows) of an fp32 [., d] matrix
                    cols = src.shape[1]
                    srcs.append(src.data_ptr() + 4 * src_row * cols)
                    dsts.append(dst.data_ptr() + 2 * dst_row * cols)
                    counts.append(nrows * cols)

                for i, blk in enumerate(self.blocks):
                    w = ws.w[i]
                    if split is None:
                        add(blk.qkv.weight, 0, w["qkv"], 0, 3 * d)
                        add(blk.up_gate.weight, 0, w["ug"], 0, 2 * W)
                    else:   # this rank's q, k and v rows; its u and gate rows
                        for part in range(3):
                            add(blk.qkv.weight, part * d + h0 * Dh, w["qkv"], part * dl, dl)
                        add(blk.up_gate.weight, u0, w["ug"], 0, Wl)
                        add(blk.up_gate.weight, W + u0, w["ug"], Wl, Wl)
                    add(blk.out_proj.weight, 0, w["out"], 0, d)
                    add(blk.down_proj.weight, 0, w["down"], 0, d)
                nw = len(srcs)
                _lib.call("engpt_cast_f32_bf16_many", (ctypes.c_void_p * nw)(*srcs), (ctypes.c_void_p * nw)(*dsts),
                          (ctypes.c_int64 * nw)(*counts), nw, st)
            scale = K.ngpt_attention_scale(Dh)
            sqrt_d = math.sqrt(float(d))
            u_mult = sqrt_d if cfg.scale_mlp_u_by_sqrt_d else 1.0
            last = len(self.blocks) - 1
            for i, blk in enumerate(self.blocks):
                if bf16:
                    wq, wo, wug, wd = ws.w[i]["qkv"], ws.w[i]["out"], ws.w[i]["ug"], ws.w[i]["down"]
                    x_in = ws.x
                else:
                    wq, wo, wug, wd = blk.qkv.weight, blk.out_proj.weight, blk.up_gate.weight, blk.down_proj.weight
                    x_in = ws.y
                    if split is not None:   # this rank's q, k, v rows and u, gate rows (fp32 mode copies them)
                        wq = torch.cat([wq[p * d + h0 * Dh:p * d + h1 * Dh] for p in range(3)])
                        wug = torch.cat([wug[u0:u1], wug[W + u0:W + u1]])
                # this rank's columns of out_proj / down_proj, its heads' s_qk rows and its units' scales
                wo_r = wo[:, h0 * Dh:h1 * Dh] if split else wo
                wd_r = wd[:, u0:u1] if split else wd
                s_qk = blk.s_qk[h0:h1]
                s_u, s_gate = blk.s_u[u0:u1], blk.s_gate[u0:u1]
                if bf16 and self.fuse_qkv and Dh in (64, 128) and dl % 256 == 0:
                    # QKV GEMM with the post-process fused into its epilogue (tcgen05): q|k|v rows are
                    # written post-processed into the same [n, 3, H, Dh] buffer
                    _lib.call("engpt_qkv_projection", x_in.data_ptr(), d, wq.data_ptr(), ws.rho.data_ptr(),
                              ws.cos.data_ptr(), ws.sin.data_ptr(), Dh // 2, s_qk.data_ptr(),
                              float(blk.qk_mult), float(cfg.norm_eps), bsz, seq_len, Hl, Dh, ws.qkv.data_ptr(), st)
                else:
                    torch.mm(x_in, wq.t(), out=ws.qkv)
                    _lib.call("engpt_qkv_postprocess", ws.qkv.data_ptr(), act, ws.rho.data_ptr(),
                              ws.cos.data_ptr(), ws.sin.data_ptr(), Dh // 2, s_qk.data_ptr(),
                              float(blk.qk_mult), float(cfg.norm_eps), bsz, seq_len, Hl, Dh, None, None, None,
                              _lib.QKV_INPLACE, st)
                if self.attn_timer is not None:
                    self.attn_timer("start")
                if self.attn_impl == _lib.ATTN_AUTO:
                    # q, k are unit vectors times the effective s_qk (the post-process above): the kernel takes
                    # its softmax offset from the per-head score bound max_i s_qk[h, i]^2 (no running max)
                    _lib.call("engpt_ngpt_attention", ws.q.data_ptr(), ws.k.data_ptr(), ws.v.data_ptr(),
                              ws.attn.data_ptr(), act, bsz, seq_len, Hl, Dh, float(scale),
                              ws.attn_strides.data_ptr(), s_qk.data_ptr(), float(blk.qk_mult), st)
                else:
                    _lib.call("engpt_causal_attention", ws.q.data_ptr(), ws.k.data_ptr(), ws.v.data_ptr(),
                              ws.attn.data_ptr(), act, bsz, seq_len, Hl, Dh, float(scale),
                              ws.attn_strides.data_ptr(), self.attn_impl, st)
                if self.attn_timer is not None:
                    self.attn_timer("stop")
                fuse_res = bf16 and self.fuse_residual and d % 256 == 0 and d <= 1024 and split is None
                if fuse_res:
                    # out_proj GEMM with the carried residual in its epilogue (tcgen05, d/256-CTA clusters):
                    # the branch never leaves the chip
                    _lib.call("engpt_gemm_carried_residual", ws.attn.data_ptr(), d, wo.data_ptr(), d, d,
                              ws.y.data_ptr(), ws.rho.data_ptr(), blk.alpha_attn_raw.data_ptr(),
                              float(blk.alpha_mult), 1, float(cfg.norm_eps), float(cfg.norm_eps),
                              float(cfg.carried_gauge_max), n, d, ws.y.data_ptr(), ws.rho.data_ptr(),
                              ws.x.data_ptr(), _lib.AUX_BF16_H, st)
                else:
                    torch.mm(ws.attn, wo_r.t(), out=ws.branch)
                    if split is not None:   # the heads' partial branches summed over the group
                        split.all_reduce_(ws.branch)
                    _lib.call("engpt_carried_residual_gauge", ws.y.data_ptr(), ws.rho.data_ptr(),
                              ws.branch.data_ptr(), act, blk.alpha_attn_raw.data_ptr(), float(blk.alpha_mult), 1,
                              float(cfg.norm_eps), float(cfg.norm_eps), float(cfg.carried_gauge_max), n, d,
                              ws.y.data_ptr(), ws.rho.data_ptr(), ws.x.data_ptr(),
                              _lib.AUX_BF16_H if bf16 else _lib.AUX_F32_H, st)
                if ws.ug is None:
                    # up/gate GEMM with the SwiGLU epilogue fused (tcgen05): the [n, 2W] projection never
                    # leaves TMEM
                    _lib.call("engpt_up_gate_swiglu", ws.x.data_ptr(), wug.data_ptr(), s_u.data_ptr(),
                              s_gate.data_ptr(), float(u_mult), float(sqrt_d), n, d, Wl,
                              ws.hidden.data_ptr(), st)
                else:
                    torch.mm(ws.x, wug.t(), out=ws.ug)
                    _lib.call("engpt_swiglu", ws.ug.data_ptr(), act, s_u.data_ptr(), s_gate.data_ptr(),
                              float(u_mult), float(sqrt_d), n, Wl, ws.hidden.data_ptr(), act, st)
                if i < last:
                    aux_mode = _lib.AUX_BF16_Y if bf16 else _lib.AUX_NONE
                else:
                    aux_mode = _lib.AUX_BF16_H if bf16 else _lib.AUX_F32_H
                if fuse_res and W % 8 == 0:
                    _lib.call("engpt_gemm_carried_residual", ws.hidden.data_ptr(), W, wd.data_ptr(), W, W,
                              ws.y.data_ptr(), ws.rho.data_ptr(), blk.alpha_mlp_raw.data_ptr(),
                              float(blk.alpha_mult), 1, float(cfg.norm_eps), float(cfg.norm_eps),
                              float(cfg.carried_gauge_max), n, d, ws.y.data_ptr(), ws.rho.data_ptr(),
                              ws.x.data_ptr(), aux_mode, st)
                else:
                    torch.mm(ws.hidden, wd_r.t(), out=ws.branch)
                    if split is not None:   # the units' partial branches summed over the group
                        split.all_reduce_(ws.branch)
                    _lib.call("engpt_carried_residual_gauge", ws.y.data_ptr(), ws.rho.data_ptr(),
                              ws.branch.data_ptr(), act, blk.alpha_mlp_raw.data_ptr(), float(blk.alpha_mult), 1,
                              float(cfg.norm_eps), float(cfg.norm_eps), float(cfg.carried_gauge_max), n, d,
                              ws.y.data_ptr(), ws.rho.data_ptr(),
                              ws.x.data_ptr() if aux_mode != _lib.AUX_NONE else None, aux_mode, st)
                if layer_callback is not None:
                    layer_callback(i, ws.y.view(bsz, seq_len, d), ws.rho.view(bsz, seq_len))
            # output head (engpt/kernels.py:209-229 with logit_scale, engpt/models.py:366-368)
            _lib.call("engpt_scale_rows_cast", self.output_emb.data_ptr(), self.s_z.data_ptr(),
                      float(self.logit_mult), cfg.vocab_size, d, ws.w_head.data_ptr(), act, st)
            # logits are computed into a [N, V_pad] buffer and returned as the [B, T, V] view of its
            # first V columns (row stride V_pad); values are those of the [N, V] product
            vp = ws.vocab_pad
            logits_buf = torch.empty(n, vp, device=dev, dtype=ws.act)
            loss = None
            if targets is not None and targets.ndim != 2:
                raise NotImplementedError("engpt_b200 implements token targets [batch, sequence] only")
            if targets is not None and bf16 and self.fuse_head and d % 8 == 0:
                # logits GEMM (tcgen05) with the per-tile log-sum-exp in its epilogue, then the merge
                t = targets.to(device=dev, dtype=torch.int64, non_blocking=True).contiguous()
                loss = torch.empty((), device=dev, dtype=torch.float32)
                _lib.call("engpt_logits_cross_entropy", ws.x.data_ptr(), ws.w_head.data_ptr(), n, d, cfg.vocab_size,
                          logits_buf.data_ptr(), vp, t.data_ptr(), ws.lse_partials().data_ptr(),
                          ws.row_loss.data_ptr(), loss.data_ptr(), st)
            else:
                torch.mm(ws.x, ws.w_head.t(), out=logits_buf)
                if targets is not None:
                    t = targets.to(device=dev, dtype=torch.int64, non_blocking=True).contiguous()
                    loss = torch.empty((), device=dev, dtype=torch.float32)
                    _lib.call("engpt_cross_entropy", logits_buf.data_ptr(), act, n, cfg.vocab_size, vp,
                              t.data_ptr(), ws.row_loss.data_ptr(), loss.data_ptr(), st)
            logits = logits_buf.view(bsz, seq_len, vp)[:, :, :cfg.vocab_size]
            if self.contiguous_logits:
                logits = logits.contiguous()
        return logits, loss

    def last_hidden(self) -> Tensor:
        """Represented state ``Y / rho`` after the last block of the latest forward, ``[B, T, d]``.

        A view of the engine's workspace (bf16 under autocast, fp32 otherwise):
        the operand of the output head, valid until the next forward.
        """
        ws = self._ws
        if ws is None:
            raise RuntimeError("last_hidden() needs a forward first")
        return ws.x.view(ws.bsz, ws.seq_len, self.cfg.n_embd)

    def forward_with_states(self, idx: Tensor, targets: Optional[Tensor] = None):
        """Forward that also returns the per-layer carried state ``[(Y, rho), ...]`` (copies)."""
        states = []
        logits, loss = self._run(idx=idx, targets=targets,
                                 layer_callback=lambda i, y, r: states.append((y.clone(), r.clone())))
        return logits, loss, states

    def parameter_norm_report(self) -> Dict[str, float]:
        """engpt/models.py:370-391."""
        with torch.no_grad():
            max_err = 0.0
            d, ff = self.cfg.n_embd, self.cfg.mlp_width
            norms = [torch.linalg.vector_norm(self.token_emb.weight, dim=-1),
                     torch.linalg.vector_norm(self.output_emb, dim=-1)]
            for b in self.blocks:
                q = b.qkv.weight
                norms += [torch.linalg.vector_norm(q[:d], dim=-1), torch.linalg.vector_norm(q[d:2 * d], dim=-1),
                          torch.linalg.vector_norm(q[2 * d:], dim=-1),
                          torch.linalg.vector_norm(b.out_proj.weight, dim=0),
                          torch.linalg.vector_norm(b.up_gate.weight[:ff], dim=-1),
                          torch.linalg.vector_norm(b.up_gate.weight[ff:], dim=-1),
                          torch.linalg.vector_norm(b.down_proj.weight, dim=0)]
            for nrm in norms:
                max_err = max(max_err, (nrm - 1.0).abs().max().item())
            return {"max_unit_norm_error": max_err}
