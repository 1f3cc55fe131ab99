"""The ThetaScan token mixer on the B200 path.

``ThetaScan(config)`` mirrors the reference public module (src/thetascan/
api.py:13-48): ``x [B,T,D] -> [B,T,D]``, ``zero_output_projection_()``,
``regularization_loss()``, and a ``_core`` submodule whose parameter and
buffer names, shapes and initialisation order follow the reference core
module (src/thetascan/_core/modules/block.py:142-333), so a reference
state dict loads unchanged and the same seed gives the same weights.

The forward of the kernel family (block.py:573-724) runs the projections as
cuBLAS GEMMs and the hot path (feature maps, multi-view scan, normalized read
and bank blend) as the sm_100a kernels of :mod:`thetascan_b200.kernel`.  With
the fused q/k/v projection, RoPE and the L2 norm of q and k run inside the
feature kernels (and their backward inside the feature backward); the other
projection layouts apply them as PyTorch f32 elementwise ops.  A bf16 input
runs bf16 streams on the tensor cores.  A float32 input runs float32
throughout, as the reference computes its fp32 configuration: the per-token
math in float32 PyTorch and every sequence read on the float32 scan kernels
(:mod:`thetascan_b200.precise`); the GN family keeps its float32 per-token
math with bf16 scan streams for either input.
"""
from __future__ import annotations

import hashlib
import math
from copy import deepcopy
from functools import lru_cache

import torch
import torch.nn as nn
import torch.nn.functional as F

from .config import ThetaScanConfig
from .kernel import KernelSpec, Prologue, kernel_core, kernel_core_qkv, kernel_core_sharded

EXPANSION_DOMAIN = "thetascan-expansion-v1"
FINGERPRINT_MAGIC = b"TSXF"
FINGERPRINT_SCHEMA = 1


def _inverse_softplus(value: float) -> float:
    return value + math.log(-math.expm1(-value))


def _domain(shape, key, role) -> bytes:
    """Versioned identity of one sign stream (block.py:67-74)."""
    return f"{EXPANSION_DOMAIN}\0{key}\0{role}\0{','.join(str(s) for s in shape)}".encode("utf-8")


def key_signs(shape, *, key: str, role: str) -> torch.Tensor:
    """+-1 signs from the low bits of SHAKE-256 over the domain (block.py:49-64)."""
    raw = bytearray(hashlib.shake_256(_domain(shape, key, role)).digest(math.prod(shape)))
    bits = torch.frombuffer(raw, dtype=torch.uint8).clone()
    return bits.bitwise_and(1).to(torch.float32).mul_(2.0).sub_(1.0).reshape(shape)


def unit_row_map(shape, *, key: str, role: str) -> torch.Tensor:
    """Uncentred sign rows scaled to unit L2 norm (block.py:117-133, center_rows=False)."""
    matrix = key_signs(shape, key=key, role=role)
    fallback = key_signs(shape, key=key, role=f"{role}-fallback")
    matrix = torch.where(matrix.norm(dim=-1, keepdim=True) > 0.0, matrix, fallback)
    return matrix / matrix.norm(dim=-1, keepdim=True)


def expansion_fingerprint(*, key: str, effective: int, expansion: int, depth: int) -> torch.Tensor:
    """40-byte persistent identity of the derived expansion maps (block.py:77-114)."""
    base = effective // expansion
    digest = hashlib.sha256()
    digest.update(b"thetascan-expansion-checkpoint\0")
    digest.update(EXPANSION_DOMAIN.encode("ascii"))
    for layer in range(depth):
        for shape, role in (((1, effective, base), f"w1-expand-layer-{layer}"),
                            ((1, base, effective), f"w2-expand-layer-{layer}")):
            descriptor = _domain(shape, key, role)
            digest.update(len(descriptor).to_bytes(8, "big"))
            digest.update(descriptor)
    encoded = FINGERPRINT_MAGIC + FINGERPRINT_SCHEMA.to_bytes(4, "big") + digest.digest()
    return torch.tensor(tuple(encoded), dtype=torch.uint8)


class _HeadLinear(nn.Module):
    """``d_model -> [B,H,T,out]`` gate projection (gates.py:6-17)."""

    def __init__(self, d_model, n_heads, out, bias_init):
        super().__init__()
        self.h, self.o = n_heads, out
        self.lin = nn.Linear(d_model, n_heads * out, bias=True)
        nn.init.zeros_(self.lin.weight)
        nn.init.constant_(self.lin.bias, bias_init)


class _OutGate(nn.Module):
    """SiLU output gate; parameters at ``ogate.g.lin`` (gates.py:34-40)."""

    def __init__(self, d_model, n_heads, d):
        super().__init__()
        self.g = _HeadLinear(d_model, n_heads, d, bias_init=1.0)


@lru_cache(maxsize=32)
def _rope_tables(T: int, rot: int, base: float, device: str):
    inv = 1.0 / (base ** (torch.arange(0, rot, 2, dtype=torch.float32, device=device) / rot))
    angles = torch.outer(torch.arange(T, dtype=torch.float32, device=device), inv)
    return angles.cos(), angles.sin()


def _rope_width(d: int, mode: str, frac: float) -> int:
    if mode == "none":
        return 0
    max_rot = d // 2 * 2
    if max_rot == 0:
        return 0
    return max_rot if mode == "full" else min(max_rot, max(2, int(d * frac) // 2 * 2))


def _rope(x: torch.Tensor, rot: int, base: float, pos0: int = 0) -> torch.Tensor:
    """Adjacent-pair rotation of the first ``rot`` channels with f32 phases
    (rope.py:57-72); ``pos0`` is the position of the first token."""
    if rot == 0:
        return x
    cos, sin = _rope_tables(pos0 + x.shape[2], rot, float(base), str(x.device))
    cos, sin = cos[pos0:], sin[pos0:]
    even, odd = x[..., 0:rot:2], x[..., 1:rot:2]
    rotated = torch.stack((even * cos - odd * sin, even * sin + odd * cos), dim=-1).flatten(-2)
    return torch.cat((rotated, x[..., rot:]), dim=-1)


def _set_param(module: nn.Module, name: str, value) -> None:
    """Point ``module.<name>`` (dotted) at ``value`` without registering it."""
    owner, _, leaf = name.rpartition(".")
    target = module.get_submodule(owner) if owner else module
    target._parameters[leaf] = value


def _l2(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``x / max(||x||, eps)`` in the input's precision (norms.py:11-12)."""
    return x / x.norm(dim=-1, keepdim=True).clamp_min(eps)


class ThetaScanCore(nn.Module):
    """Parameters and forward of one mixer (reference block.ThetaScan)."""

    def __init__(self, cfg: ThetaScanConfig):
        super().__init__()
        self.cfg = cfg
        reason = cfg.unsupported_reason()
        if reason is not None:
            raise NotImplementedError(f"thetascan_b200: {reason}")
        D, H, d = cfg.d_model, cfg.n_heads, cfg.resolved_head_dim
        m = cfg.memory_width
        k = cfg.kernel
        self.n_heads, self.head_dim, self.mem_hidden = H, d, m
        kernel = cfg.family == "kernel"
        # Control parameters, in the reference's construction order (the GN
        # family has none).
        if kernel and k.kernel_sharpness_mode == "learned_per_head":
            self.kernel_sharpness_raw = nn.Parameter(torch.full((H,), _inverse_softplus(float(k.kernel_sharpness))))
        elif kernel and k.kernel_sharpness_mode == "learned_per_feature":
            self.kernel_sharpness_raw = nn.Parameter(
                torch.full((H, m), _inverse_softplus(float(k.kernel_sharpness))))
        else:
            self.register_parameter("kernel_sharpness_raw", None)
        self.kernel_score_bias = nn.Parameter(torch.zeros(H, m)) if kernel and k.score_bias else None
        if kernel and k.relu2_threshold_mode == "learned_per_head":
            self.kernel_relu2_threshold = nn.Parameter(torch.zeros(H))
        else:
            self.register_parameter("kernel_relu2_threshold", None)
        if kernel and k.sparsity != "none":
            # relative-to-maximum cutoff rho = sigmoid(raw) (block.py:167-180)
            rho0 = float(k.relative_threshold_init)
            self.kernel_relative_threshold_raw = nn.Parameter(torch.full((H,), math.log(rho0 / (1.0 - rho0))))
        else:
            self.register_parameter("kernel_relative_threshold_raw", None)
        if kernel and k.sparsity == "relative_st_blend":
            self.kernel_sparse_blend_raw = nn.Parameter(torch.full((H,), float(k.sparse_blend_init)))
        else:
            self.register_parameter("kernel_sparse_blend_raw", None)
        if kernel and k.bspline_scale_mode == "learned_per_head":
            self.bspline_scale_raw = nn.Parameter(torch.full((H,), _inverse_softplus(float(k.bspline_scale))))
        else:
            self.register_parameter("bspline_scale_raw", None)
        # Projections (block.py:186-207).
        if cfg.key_value_heads is not None:
            G = cfg.key_value_heads
            self.proj_qkv = None
            self.proj_q = nn.Linear(D, H * d, bias=False)
            self.proj_k = nn.Linear(D, G * d, bias=False)
            self.proj_v = nn.Linear(D, G * d, bias=False)
        elif cfg.share_key_query:
            self.proj_qkv = None
            self.proj_q1 = nn.Linear(D, d, bias=False)
            self.proj_k1 = nn.Linear(D, d, bias=False)
            self.proj_v = nn.Linear(D, H * d, bias=False)
            self.kq_bias = nn.Parameter(torch.zeros(2, H, d))
        else:
            self.proj_qkv = nn.Linear(D, 3 * H * d, bias=False)
        self.proj_out = nn.Linear(H * d, D, bias=False)
        # Memory net theta0 (block.py:210-301): one (W1, W2, Wg) per layer,
        # drawn in the reference's order (every W1, every W2, every Wg).
        L = cfg.depth
        projections = m // k.bspline_basis_count if kernel and k.feature_map == "projected_bspline" else m
        self.W1 = nn.ParameterList([nn.Parameter(torch.randn(H, projections, d) / math.sqrt(d)) for _ in range(L)])
        self.W2 = nn.ParameterList([nn.Parameter(torch.zeros(H, d, m)) for _ in range(L)])
        if not kernel and cfg.gn.nonlinearity == "swiglu":
            # swiglu gate branch, at the effective width (never expanded)
            self.Wg = nn.ParameterList([nn.Parameter(torch.randn(H, m, d) / math.sqrt(d)) for _ in range(L)])
        elif not kernel and cfg.gn.nonlinearity == "relu2_threshold":
            # GN learned threshold tau rides the Wg slot (block.py:231-235), zero-init
            self.Wg = nn.ParameterList([nn.Parameter(torch.zeros(H, m, 1)) for _ in range(L)])
        else:
            self.Wg = None
        self.register_buffer("_expansion_fingerprint", None)
        self._expanded = cfg.feature_expansion > 1
        if self._expanded:
            b = m // cfg.feature_expansion
            self.W1 = nn.ParameterList([nn.Parameter(torch.randn(H, b, d) / math.sqrt(d)) for _ in range(L)])
            self.W2 = nn.ParameterList([nn.Parameter(torch.zeros(H, d, b)) for _ in range(L)])
            for layer in range(L):
                self.register_buffer(f"_expand_w1_{layer}", unit_row_map(
                    (1, m, b), key=cfg.expansion_key, role=f"w1-expand-layer-{layer}"), persistent=False)
                self.register_buffer(f"_expand_w2_{layer}", unit_row_map(
                    (1, b, m), key=cfg.expansion_key, role=f"w2-expand-layer-{layer}"), persistent=False)
            self._expansion_fingerprint = expansion_fingerprint(
                key=cfg.expansion_key, effective=m, expansion=cfg.feature_expansion, depth=L)
        self.vmlp_in = self.vmlp_out = None
        if k.value_representation == "value_mlp":
            vh = max(1, int(k.value_mlp_multiplier * d))
            self.vmlp_in = nn.Linear(d, vh)
            self.vmlp_out = nn.Linear(vh, d)
            nn.init.zeros_(self.vmlp_out.weight)
            nn.init.zeros_(self.vmlp_out.bias)
        self.ogate = _OutGate(D, H, d) if cfg.output_gate else None
        # Temporal bank (block.py:313-330).
        t = cfg.temporal
        self.branches = t.recency_branches if t.mode == "bank" else 0
        if t.mode == "bank":
            alphas = t.resolved_retentions()
            if t.recency_branches == 1:
                self.fade_alpha = nn.Parameter(torch.full((H,), math.log(alphas[0] / (1.0 - alphas[0]))))
                self.fade_eta = nn.Parameter(torch.zeros(H))
            else:
                raw = [math.log(a / (1.0 - a)) for a in alphas]
                self.fade_alpha = nn.Parameter(torch.tensor(raw).view(-1, 1).expand(-1, H).clone())
                self.fade_eta = nn.Parameter(torch.zeros(t.recency_branches, H))
        else:
            self.fade_alpha = None
            self.fade_eta = None
        self.spec = KernelSpec(
            kind=k.feature_map, mode=("sum" if t.mode == "sum" else t.bank_mode),
            eps=1e-6, gain=float(k.kernel_sharpness), basis=k.bspline_basis_count,
            bound=float(k.bspline_bound), spline_scale=float(k.bspline_scale), read=k.read_normalization,
            sparsity=k.sparsity, temperature=float(k.threshold_temperature))
        self._rot = _rope_width(d, cfg.rope.mode, cfg.rope.fraction)

    # -------------------------------------------------------------- helpers

    def _forward_gn(self, x, shard):
        """GN family: f32 projections on TF32 tensor cores, q/k preparation
        and the GN core on the row kernels, every sequence read on the scan
        kernels (:mod:`thetascan_b200.gn`)."""
        from .gn import gn_core, per_token, tf32_linear
        B, T, _ = x.shape
        H, d = self.n_heads, self.head_dim
        # The write's solve divides by ||k||^2-weighted terms and amplifies
        # rounding of its inputs (bf16 projections move the input gradient by
        # ~3%), so projections, q/k preparation and the per-token math stay
        # f32; only the scan streams are bf16.
        xf = x.float()
        rot, base = self._rot, self.cfg.rope.base
        gn = self.cfg.gn
        eps = 1e-6 if gn.damping is None else float(gn.damping)
        # Deeper nets and swiglu (gn_deep) keep every product in plain f32:
        # their retention gradients amplify a 2^-11 perturbation of q and k by
        # ~40x, beyond what TF32 projections leave within tolerance.
        # Sequence shards take the same path, every read entering with the
        # earlier shards' state.
        deep = self.cfg.depth > 1 or gn.nonlinearity == "swiglu" or shard is not None
        lin = F.linear if deep else tf32_linear
        pos0 = 0 if shard is None else shard.rank * T
        if self.cfg.key_value_heads is None and not self.cfg.share_key_query:
            # fused projection, then RoPE + L2 of q and k in one row kernel
            from . import ops  # noqa: F401  (registers the operators)
            qkv = lin(xf, self.proj_qkv.weight)
            if rot:
                cos, sin = _rope_tables(pos0 + T, rot, float(base), str(x.device))
                cos, sin = cos[pos0:], sin[pos0:]
            else:
                cos = sin = qkv.new_empty(0)
            q, k, v = torch.ops.thetascan_b200.gn_prep_fwd(qkv, cos, sin, rot, H, eps)
        else:
            names = [n for n, _ in self.named_parameters() if n.startswith("proj_") or n == "kq_bias"]
            params = dict(self.named_parameters())

            def qkv_fn(xx, *ws):
                # the module's projection with its weights passed in (so that
                # the TF32 recomputation differentiates them)
                saved = {n: params[n] for n in names}
                try:
                    for n, w in zip(names, ws):
                        _set_param(self, n, w)
                    q, k, v = self.project(xx)
                finally:
                    for n in names:
                        _set_param(self, n, saved[n])
                return q.contiguous(), k.contiguous(), v.contiguous()

            ws = [params[n] for n in names]
            q, k, v = qkv_fn(xf, *ws) if deep else per_token(qkv_fn, xf, *ws)
            q, k = _l2(_rope(q, rot, base, pos0), eps), _l2(_rope(k, rot, base, pos0), eps)
        if self.vmlp_in is not None:
            v = v + self.vmlp_out(F.silu(self.vmlp_in(v)))
        log_alphas, etas = self.fade()
        nonlin = "relu2" if gn.nonlinearity == "relu2_threshold" else gn.nonlinearity
        mode = self.spec.mode if log_alphas is not None else "sum"
        if not deep:
            W1, W2 = self.effective_weights()
            y = gn_core(q, k, v, W1, W2, None if self.Wg is None else self.Wg[0], nonlin=nonlin,
                        read_norm=gn.read_normalization != "none",
                        read_norm_w1=gn.read_normalization == "both_feature_mass",
                        log_alphas=log_alphas, etas=etas, mode=mode, eps=eps, steps=gn.jacobian_steps)
        else:
            # deeper nets, the swiglu activation and sequence shards (gn_deep:
            # per-token maps in f32 PyTorch, every read on the scan kernels)
            from .gn_deep import gn_deep
            layers = [self.effective_weights(l) + (None if self.Wg is None else self.Wg[l],)
                      for l in range(self.cfg.depth)]
            y = gn_deep(q, k, v, layers, nonlin=nonlin, thresholded=gn.nonlinearity == "relu2_threshold",
                        read_norm=gn.read_normalization != "none",
                        read_norm_w1=gn.read_normalization == "both_feature_mass",
                        log_alphas=log_alphas, etas=etas, mode=mode, eps=eps, steps=gn.jacobian_steps,
                        shard=shard)
        y = y.transpose(1, 2)
        if self.ogate is not None:
            g = lin(xf, self.ogate.g.lin.weight, self.ogate.g.lin.bias)
            y = F.silu(g).view(B, T, H, d) * y
        y = lin(y.reshape(B, T, H * d), self.proj_out.weight)
        return y.to(x.dtype)

    def _forward_f32(self, x, shard):
        """Kernel family on a float32 input: float32 throughout, the sequence
        reads on the float32 scan kernels (:mod:`thetascan_b200.precise`); on
        a sequence shard every read enters with the earlier shards' state."""
        from .precise import kernel_core_f32
        B, T, _ = x.shape
        H, d = self.n_heads, self.head_dim
        rot, base = self._rot, self.cfg.rope.base
        pos0 = 0 if shard is None else shard.rank * T
        q, k, v = self.project(x)
        q, k = _l2(_rope(q, rot, base, pos0)), _l2(_rope(k, rot, base, pos0))
        if self.vmlp_in is not None:
            v = v + self.vmlp_out(F.silu(self.vmlp_in(v)))
        W1, W2 = self.effective_weights()
        log_alphas, etas = self.fade()
        y = kernel_core_f32(q, k, v.contiguous(), W1, W2, self.spec, log_alphas=log_alphas, etas=etas, shard=shard,
                            **self.kernel_controls()).transpose(1, 2)
        if self.ogate is not None:
            lin = self.ogate.g.lin
            y = y * F.silu(F.linear(x, lin.weight, lin.bias).view(B, T, H, d))
        return F.linear(y.reshape(B, T, H * d), self.proj_out.weight)

    def _fused_shards(self) -> bool:
        """Whether sequence shards run the fused bf16 core (two scan stages
        around one exchange, kernel.kernel_core_sharded): the fused q/k/v
        projection, no value MLP, the key-mass read, the plain sum or a fast
        bank, no relative sparsity."""
        return (self.proj_qkv is not None and self.vmlp_in is None and self.spec.read == "key_mass"
                and self.spec.mode != "stale" and self.spec.sparsity == "none")

    def effective_weights(self, layer: int = 0):
        """``U W1`` and ``W2 D`` of one layer (block.py:546-567)."""
        W1, W2 = self.W1[layer], self.W2[layer]
        if self._expanded:
            W1 = torch.matmul(getattr(self, f"_expand_w1_{layer}"), W1)
            W2 = torch.matmul(W2, getattr(self, f"_expand_w2_{layer}"))
        return W1, W2

    def fade(self):
        """Per-branch ``log_alpha = -softplus(-raw)`` and blends, ``[J,H]``."""
        if self.fade_alpha is None:
            return None, None
        raw, eta = self.fade_alpha, self.fade_eta
        if raw.ndim == 1:
            raw, eta = raw.unsqueeze(0), eta.unsqueeze(0)
        if self.cfg.temporal.blend_mode == "tanh":
            eta = torch.tanh(eta)
        return -F.softplus(-raw), eta

    def kernel_controls(self):
        gain = None if self.kernel_sharpness_raw is None else \
            F.softplus(self.kernel_sharpness_raw).clamp_min(torch.finfo(torch.float32).tiny)
        scale = None if self.bspline_scale_raw is None else \
            F.softplus(self.bspline_scale_raw).clamp_min(torch.finfo(torch.float32).tiny)
        ctl = dict(threshold=self.kernel_relu2_threshold, score_bias=self.kernel_score_bias, gain=gain,
                   spline_scale=scale)
        if self.kernel_relative_threshold_raw is not None:
            ctl["relative_threshold"] = torch.sigmoid(self.kernel_relative_threshold_raw)
        if self.kernel_sparse_blend_raw is not None:
            # forward value clamp(raw, 0, 1), gradient through sigmoid(raw) (block.py:427-438)
            raw = self.kernel_sparse_blend_raw
            surrogate = torch.sigmoid(raw)
            ctl["sparse_blend"] = raw.clamp(0.0, 1.0).detach() + surrogate - surrogate.detach()
        return ctl

    def project(self, x):
        """q, k, v ``[B,H,T,d]`` in the stream dtype (block.py:577-594)."""
        cfg = self.cfg
        B, T, _ = x.shape
        H, d = self.n_heads, self.head_dim
        dt = x.dtype
        if cfg.key_value_heads is not None:
            G = cfg.key_value_heads
            q = F.linear(x, self.proj_q.weight.to(dt)).view(B, T, H, d).transpose(1, 2)
            k = F.linear(x, self.proj_k.weight.to(dt)).view(B, T, G, d).transpose(1, 2)
            v = F.linear(x, self.proj_v.weight.to(dt)).view(B, T, G, d).transpose(1, 2)
            return q, k.repeat_interleave(H // G, dim=1), v.repeat_interleave(H // G, dim=1)
        if cfg.share_key_query:
            bias = self.kq_bias.to(dt)
            q = F.linear(x, self.proj_q1.weight.to(dt)).unsqueeze(1) + bias[0][None, :, None, :]
            k = F.linear(x, self.proj_k1.weight.to(dt)).unsqueeze(1) + bias[1][None, :, None, :]
            v = F.linear(x, self.proj_v.weight.to(dt)).view(B, T, H, d).transpose(1, 2)
            return q, k, v
        qkv = F.linear(x, self.proj_qkv.weight.to(dt))
        q, k, v = qkv.view(B, T, 3, H, d).permute(2, 0, 3, 1, 4)
        return q, k, v

    def prepare_qk(self, x):
        """RoPE then L2 norm with f32 arithmetic, back to bf16 (block.py:595-599)."""
        x = _rope(x.float(), self._rot, self.cfg.rope.base)
        return (x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)).to(torch.bfloat16).contiguous()

    def forward(self, x: torch.Tensor, shard=None) -> torch.Tensor:
        """``x [B,T,D]``; with ``shard`` (a :class:`thetascan_b200.seqpar.SeqShard`)
        ``x`` is this rank's contiguous T-slice of longer sequences, and the
        chunk states of the earlier slices arrive through one exchange."""
        if not x.is_cuda:
            raise RuntimeError("thetascan_b200 requires a CUDA input")
        if torch.is_autocast_enabled("cuda"):
            # The mixer picks its own precisions (bf16 streams on the tensor
            # cores with f32 states; the GN family's per-token math in f32),
            # so autocast is off inside; under a bf16 autocast a float32 input
            # of the kernel family takes the bf16 path.
            to_bf16 = (self.cfg.family != "gn" and x.dtype == torch.float32
                       and torch.get_autocast_dtype("cuda") == torch.bfloat16)
            with torch.autocast("cuda", enabled=False):
                return self.forward(x.to(torch.bfloat16) if to_bf16 else x, shard)
        if self.cfg.family == "gn":
            return self._forward_gn(x, shard)
        if x.dtype == torch.float32:
            return self._forward_f32(x, shard)
        if shard is not None and not self._fused_shards():
            # sequence shards of the other views and reads: the float32 path,
            # each scan entering with the earlier shards' state
            return self._forward_f32(x.float(), shard).to(x.dtype)
        B, T, _ = x.shape
        H, d = self.n_heads, self.head_dim
        out_dtype = x.dtype
        xb = x.to(torch.bfloat16)
        W1, W2 = self.effective_weights()
        log_alphas, etas = self.fade()
        if shard is not None:
            qkv = F.linear(xb, self.proj_qkv.weight.to(torch.bfloat16))
            pos0 = shard.rank * T
            cos = sin = None
            if self._rot:
                cos, sin = _rope_tables(pos0 + T, self._rot, float(self.cfg.rope.base), str(x.device))
            prologue = Prologue(self._rot, cos, sin, 1e-6, pos0)
            y = kernel_core_sharded(qkv, H, W1, W2, self.spec, prologue, shard, log_alphas=log_alphas, etas=etas,
                                    **self.kernel_controls())
        elif self.proj_qkv is not None and self.vmlp_in is None and self.spec.read == "key_mass":
            # Fused projection layout: RoPE and the L2 norm run inside the
            # feature kernels, v is read from the projection in place.
            qkv = F.linear(xb, self.proj_qkv.weight.to(torch.bfloat16))
            cos = sin = None
            if self._rot:
                cos, sin = _rope_tables(T, self._rot, float(self.cfg.rope.base), str(x.device))
            prologue = Prologue(self._rot, cos, sin, 1e-6)
            y = kernel_core_qkv(qkv, H, W1, W2, self.spec, prologue, log_alphas=log_alphas, etas=etas,
                                **self.kernel_controls())
        else:
            q, k, v = self.project(xb)
            q, k = self.prepare_qk(q), self.prepare_qk(k)
            if self.vmlp_in is not None:
                v = v + self.vmlp_out(F.silu(self.vmlp_in(v.float()))).to(v.dtype)
            v = v.contiguous()
            y = kernel_core(q, k, v, W1, W2, self.spec, log_alphas=log_alphas, etas=etas,
                            **self.kernel_controls())
        if self.ogate is not None:
            lin = self.ogate.g.lin
            gate = F.linear(xb, lin.weight.to(torch.bfloat16), lin.bias.to(torch.bfloat16))
            y = y * F.silu(gate.view(B, T, H, d))
        y = F.linear(y.reshape(B, T, H * d), self.proj_out.weight.to(torch.bfloat16))
        return y.to(out_dtype)


class ThetaScan(nn.Module):
    """Public mixer: ``x [B,T,D] -> [B,T,D]`` (reference api.py:13-48)."""

    def __init__(self, config: ThetaScanConfig):
        super().__init__()
        self.config = deepcopy(config)
        self.config.validate()
        self._core = ThetaScanCore(self.config)
        if self.config.family == "kernel" and not self.config.kernel.feature_parameters_trainable:
            for p in (self._core.W1[0], self._core.kernel_sharpness_raw, self._core.kernel_score_bias,
                      self._core.kernel_relu2_threshold, self._core.bspline_scale_raw):
                if p is not None:
                    p.requires_grad_(False)

    def forward(self, x: torch.Tensor, shard=None) -> torch.Tensor:
        return self._core(x, shard)

    def zero_output_projection_(self) -> "ThetaScan":
        nn.init.zeros_(self._core.proj_out.weight)
        return self

    def regularization_loss(self) -> torch.Tensor:
        """Optional decorrelation penalty of theta0 (block.py:496-544)."""
        cfg = self.config.regularization
        out = torch.zeros((), device=self._core.W2[0].device)
        mats = [self._core.W1[0], self._core.W2[0]]
        if cfg.feature_weight:
            acc = 0.0
            eligible = [W for W in mats if W.shape[-2] > 1]
            for W in eligible:
                Wn = W / W.norm(dim=-1, keepdim=True).clamp_min(1e-6)
                G = Wn @ Wn.transpose(-1, -2)
                r = G.shape[-1]
                acc = acc + (G * (1.0 - torch.eye(r, device=G.device))).square().sum() / (G.shape[0] * r * (r - 1))
            if eligible:
                out = out + cfg.feature_weight * acc / len(eligible)
        if cfg.head_weight and self.config.n_heads > 1:
            acc = 0.0
            for W in mats:
                V = W.flatten(1)
                Vn = V / V.norm(dim=-1, keepdim=True).clamp_min(1e-6)
                Gh = Vn @ Vn.t()
                n = Gh.shape[0]
                acc = acc + (Gh * (1.0 - torch.eye(n, device=Gh.device))).square().sum() / (n * (n - 1))
            out = out + cfg.head_weight * acc / len(mats)
        return out
