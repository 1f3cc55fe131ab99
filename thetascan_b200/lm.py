"""A small hybrid language model around the b200 mixer (baseline config 5).

The reference trains its mixers inside an external GPT host that it does not
ship (benchmarks/parameter-golf/prepare_harness.py:649-740 patches
``build_mixer`` and ``Block`` into a cloned training script).  This module is
a self-contained host of the same shape -- for exercising the mixer under
autograd, bf16 autocast, data-parallel training and AdamW, and for timing a
whole training step:

* token embedding of a 1024-entry vocabulary, tied to the output head;
* nine pre-norm residual blocks ``x + mix(norm(x))``, ``x + mlp(norm(x))``
  with RMS norms, d_model 512, 8 heads, MLP hidden width 2 x d_model
  (squared-ReLU);
* the two middle blocks mix with a ThetaScan-GN mixer of this package
  (``thetascan_b200.ThetaScan``; the expanded GN layout of the reference's
  ``gn_expanded_reference_v0_1`` preset, config.py:832-862: shared k/q
  projection, learned relu2 threshold, 2x random feature expansion,
  two-stage feature-mass read, one fast recency branch -- at memory
  multiplier 2, m = 256, the widest the scan kernels take), the others with
  causal softmax attention (``scaled_dot_product_attention``, RoPE on q/k).

The mixer's output projection starts at zero, as the reference's adapter
initialises it (thetascan_benchmark_adapter.py:83).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .config import GNConfig, RoPEConfig, TemporalConfig, ThetaScanConfig
from .mixer import ThetaScan


def gn_mixer_config(d_model: int = 512, n_heads: int = 8, memory_multiplier: int = 2) -> ThetaScanConfig:
    """The expanded GN mixer layout of config 5 at memory multiplier 2."""
    return ThetaScanConfig(
        d_model=d_model, n_heads=n_heads, memory_multiplier=memory_multiplier, feature_expansion=2,
        share_key_query=True, output_gate=False, family="gn",
        gn=GNConfig(nonlinearity="relu2_threshold", jacobian_steps=1, read_normalization="both_feature_mass"),
        rope=RoPEConfig(mode="partial", fraction=0.5, base=10_000.0),
        temporal=TemporalConfig(mode="bank", bank_mode="fast", recency_branches=1, retention_inits=(0.9,),
                                blend_mode="free"))


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


def _rope(x, base: float = 10_000.0):
    """Adjacent-pair rotation of all channels of ``x [B,H,T,d]`` (f32 phases)."""
    B, H, T, d = x.shape
    inv = 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float32, device=x.device) / d))
    ang = torch.outer(torch.arange(T, dtype=torch.float32, device=x.device), inv)
    cos, sin = ang.cos().to(x.dtype), ang.sin().to(x.dtype)
    even, odd = x[..., 0::2], x[..., 1::2]
    return torch.stack((even * cos - odd * sin, even * sin + odd * cos), dim=-1).flatten(-2)


class CausalAttention(nn.Module):
    def __init__(self, d_model: int, n_heads: int):
        super().__init__()
        self.n_heads = n_heads
        self.qkv = nn.Linear(d_model, 3 * d_model, bias=False)
        self.out = nn.Linear(d_model, d_model, bias=False)

    def forward(self, x):
        B, T, D = x.shape
        q, k, v = self.qkv(x).view(B, T, 3, self.n_heads, D // self.n_heads).permute(2, 0, 3, 1, 4)
        y = F.scaled_dot_product_attention(_rope(q), _rope(k), v, is_causal=True)
        return self.out(y.transpose(1, 2).reshape(B, T, D))


class MLP(nn.Module):
    def __init__(self, d_model: int, ratio: int):
        super().__init__()
        self.up = nn.Linear(d_model, ratio * d_model, bias=False)
        self.down = nn.Linear(ratio * d_model, d_model, bias=False)

    def forward(self, x):
        return self.down(F.relu(self.up(x)).square())


class Block(nn.Module):
    def __init__(self, d_model: int, n_heads: int, mlp_ratio: int, mixer: nn.Module):
        super().__init__()
        self.norm1, self.norm2 = RMSNorm(d_model), RMSNorm(d_model)
        self.mix = mixer
        self.mlp = MLP(d_model, mlp_ratio)

    def forward(self, x):
        x = x + self.mix(self.norm1(x))
        return x + self.mlp(self.norm2(x))


class HybridLM(nn.Module):
    """Nine-block hybrid LM; blocks in ``mixer_layers`` use the GN mixer."""

    def __init__(self, vocab: int = 1024, d_model: int = 512, n_layers: int = 9, n_heads: int = 8,
                 mlp_ratio: int = 2, mixer_layers=(3, 4), mixer_config: ThetaScanConfig | None = None,
                 mixer_factory=None):
        """``mixer_factory(config)`` builds a mixer module (default: this
        package's ThetaScan; a test passes the reference's own to compare)."""
        super().__init__()
        self.embed = nn.Embedding(vocab, d_model)
        nn.init.normal_(self.embed.weight, std=0.02)
        cfg = mixer_config if mixer_config is not None else gn_mixer_config(d_model, n_heads)
        factory = mixer_factory if mixer_factory is not None else ThetaScan
        blocks = []
        for i in range(n_layers):
            if i in mixer_layers:
                mixer = factory(cfg)
                mixer.zero_output_projection_()
            else:
                mixer = CausalAttention(d_model, n_heads)
            blocks.append(Block(d_model, n_heads, mlp_ratio, mixer))
        self.blocks = nn.ModuleList(blocks)
        self.norm = RMSNorm(d_model)
        # residual-branch outputs of the attention and MLP blocks (the mixers
        # keep their zero output projection)
        for name, p in self.named_parameters():
            if name.endswith("mlp.down.weight") or name.endswith("mix.out.weight"):
                nn.init.normal_(p, std=0.02 / math.sqrt(2 * n_layers))

    def forward(self, tokens):
        x = self.embed(tokens)
        for block in self.blocks:
            x = block(x)
        return F.linear(self.norm(x), self.embed.weight)

    def loss(self, tokens):
        """Next-token cross entropy of ``tokens [B,T]`` (predicting 1..T-1)."""
        logits = self(tokens[:, :-1])
        return F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), tokens[:, 1:].reshape(-1))
