"""Blocks and the language model around KulaMamba (drop-in for ``mamba3.block``).

This is the harness the decode and LM configs run through; it mirrors the
reference's module structure, names and init order (mamba3/block.py:16-231) so
seeded weights and state dicts match.  The MLP's GEMMs are cuBLAS; at inference the norms,
the SwiGLU activation and the scaled residuals are one library kernel each (torch ops when
autograd runs through them); the SSM layer is ``mamba3_b200.mamba3.KulaMamba``.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as grad_checkpoint

from . import ops
from .mamba3 import KulaMamba, RMSNorm


def _residual(x, h, scale):
    """x + h * scale (the blocks' scaled residuals): one kernel when no autograd goes through."""
    return ops.scaled_add(x, h, scale) if ops.kernel_ok(x, h) else x + h * scale


class SwiGLU(nn.Module):
    """w_down(silu(w_gate x) * w_up x)  (mamba3/block.py:16-26)."""

    def __init__(self, d_model: int, d_ff: int | None = None, bias: bool = False):
        super().__init__()
        d_ff = d_ff or int(d_model * 8 / 3 / 64 + 1) * 64
        self.w_gate = nn.Linear(d_model, d_ff, bias=bias)
        self.w_up = nn.Linear(d_model, d_ff, bias=bias)
        self.w_down = nn.Linear(d_ff, d_model, bias=bias)

    def _stacked(self):
        """[w_gate; w_up] (and biases) as one weight, rebuilt whenever either changes."""
        wg, wu = self.w_gate.weight, self.w_up.weight
        key = (wg.data_ptr(), wg._version, wu.data_ptr(), wu._version, wg.dtype, wg.device)
        if getattr(self, "_gu_key", None) != key:
            self._gu_w = torch.cat([wg.detach(), wu.detach()], 0)
            self._gu_b = (torch.cat([self.w_gate.bias.detach(), self.w_up.bias.detach()], 0)
                          if self.w_gate.bias is not None else None)
            self._gu_key = key
        return self._gu_w, self._gu_b

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        d_ff = self.w_gate.out_features
        if (ops.kernel_ok(x) and d_ff % 8 == 0
                and not (torch.is_grad_enabled() and any(p.requires_grad for p in self.parameters()))):
            # inference: the gate and up projections as one GEMM over the stacked weights
            w, b = self._stacked()
            return self.w_down(ops.swiglu_rows(F.linear(x, w, b)))
        g, u = self.w_gate(x), self.w_up(x)
        a = ops.swiglu_act(g, u) if ops.kernel_ok(g, u) else F.silu(g) * u
        return self.w_down(a)


class KulaMambaBlock(nn.Module):
    """Pre-norm SSM + optional SwiGLU with scaled residuals (mamba3/block.py:29-107)."""

    def __init__(
        self,
        d_model: int,
        d_state: int = 128,
        expand: int = 2,
        headdim: int = 64,
        ngroups: int | None = None,
        mimo_rank: int = 2,
        chunk_size: int = 64,
        use_mlp: bool = True,
        mlp_expand: float = 2.667,
        norm_eps: float = 1e-5,
        bias: bool = False,
        residual_scale: float = 1.0,
        gradient_checkpointing: bool = False,
        use_trapezoidal: bool = True,
        use_complex_ssm: bool = True,
    ):
        super().__init__()
        self.residual_scale = residual_scale
        self.gradient_checkpointing = gradient_checkpointing
        self.ssm_norm = RMSNorm(d_model, eps=norm_eps)
        self.ssm = KulaMamba(d_model=d_model, d_state=d_state, expand=expand, headdim=headdim, ngroups=ngroups,
                             mimo_rank=mimo_rank, chunk_size=chunk_size, bias=bias,
                             use_trapezoidal=use_trapezoidal, use_complex_ssm=use_complex_ssm)
        self.use_mlp = use_mlp
        if use_mlp:
            d_ff = int(d_model * mlp_expand / 64 + 1) * 64
            self.mlp_norm = RMSNorm(d_model, eps=norm_eps)
            self.mlp = SwiGLU(d_model, d_ff, bias=bias)

    def _mlp_residual(self, x):
        if self.use_mlp:
            if self.gradient_checkpointing and self.training:
                m = grad_checkpoint(lambda t: self.mlp(self.mlp_norm(t)), x, use_reentrant=False)
            else:
                m = self.mlp(self.mlp_norm(x))
            x = _residual(x, m, self.residual_scale)
        return x

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.gradient_checkpointing and self.training:
            h = grad_checkpoint(lambda t: self.ssm(self.ssm_norm(t)), x, use_reentrant=False)
        else:
            h = self.ssm(self.ssm_norm(x))
        return self._mlp_residual(_residual(x, h, self.residual_scale))

    def step(self, x, ssm_state):
        h, new_state = self.ssm.step(self.ssm_norm(x), ssm_state)
        return self._mlp_residual(_residual(x, h, self.residual_scale)), new_state

    def prefill(self, x, compact_state=False):
        h, state = self.ssm.prefill(self.ssm_norm(x), compact_state=compact_state)
        return self._mlp_residual(_residual(x, h, self.residual_scale)), state


class KulaMambaLM(nn.Module):
    """Embedding -> n_layers blocks -> RMSNorm -> tied lm_head (mamba3/block.py:110-231)."""

    def __init__(
        self,
        vocab_size: int,
        d_model: int = 768,
        n_layers: int = 12,
        d_state: int = 128,
        expand: int = 2,
        headdim: int = 64,
        ngroups: int | None = None,
        mimo_rank: int = 2,
        chunk_size: int = 64,
        use_mlp: bool = True,
        tie_weights: bool = True,
        norm_eps: float = 1e-5,
        bias: bool = False,
        residual_scale: str = "depth",
        gradient_checkpointing: bool = False,
        use_trapezoidal: bool = True,
        use_complex_ssm: bool = True,
    ):
        super().__init__()
        self.d_model = d_model
        self.n_layers = n_layers
        r_scale = 1.0 / math.sqrt(2 * n_layers) if residual_scale == "depth" else 1.0
        self.embedding = nn.Embedding(vocab_size, d_model)
        self.layers = nn.ModuleList([
            KulaMambaBlock(d_model=d_model, d_state=d_state, expand=expand, headdim=headdim, ngroups=ngroups,
                           mimo_rank=mimo_rank, chunk_size=chunk_size, use_mlp=use_mlp, norm_eps=norm_eps, bias=bias,
                           residual_scale=r_scale, gradient_checkpointing=gradient_checkpointing,
                           use_trapezoidal=use_trapezoidal, use_complex_ssm=use_complex_ssm)
            for _ in range(n_layers)
        ])
        self.norm = RMSNorm(d_model, eps=norm_eps)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)
        if tie_weights:
            self.lm_head.weight = self.embedding.weight
        self._init_weights()

    def _init_weights(self):
        """N(0, 0.02) for embedding and Linears, then the KulaMamba init again (mamba3/block.py:166-176)."""
        nn.init.normal_(self.embedding.weight, std=0.02)
        for m in self.modules():
            if isinstance(m, nn.Linear) and m is not self.lm_head:
                nn.init.normal_(m.weight, std=0.02)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
        for m in self.modules():
            if isinstance(m, KulaMamba):
                m._init_weights(dt_min=0.001, dt_max=0.1)

    def _forward_fused(self, x):
        """Inference forward with the residual adds inside the stack fused into the norm that
        follows each (ops.add_rmsnorm: the same stored values as the residual kernel then the norm
        kernel); the final norm runs as its module, so hooks on it still see its output."""
        n = self.layers[0].ssm_norm(x)
        last = len(self.layers) - 1
        for i, blk in enumerate(self.layers):
            h = blk.ssm(n)
            if blk.use_mlp:
                x, n1 = ops.add_rmsnorm(x, h, blk.residual_scale, blk.mlp_norm.weight, blk.mlp_norm.eps)
                h = blk.mlp(n1)
            if i < last:
                nxt = self.layers[i + 1].ssm_norm
                x, n = ops.add_rmsnorm(x, h, blk.residual_scale, nxt.weight, nxt.eps)
            else:
                n = self.norm(_residual(x, h, blk.residual_scale))
        return n

    def forward(self, input_ids, labels=None):
        x = self.embedding(input_ids)
        if (ops.kernel_ok(x) and x.dtype in (torch.bfloat16, torch.float16) and x.shape[-1] % 8 == 0
                and x.shape[-1] <= 2048 and not torch.is_grad_enabled()):
            logits = self.lm_head(self._forward_fused(x))
        else:
            for layer in self.layers:
                x = layer(x)
            logits = self.lm_head(self.norm(x))
        result = {"logits": logits}
        if labels is not None:
            result["loss"] = F.cross_entropy(logits[:, :-1].reshape(-1, logits.size(-1)), labels[:, 1:].reshape(-1))
        return result

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens=100, temperature=1.0, top_k=None):
        """Prefill every layer, then decode token by token (mamba3/block.py:195-231)."""
        x = self.embedding(input_ids)
        states = []
        for layer in self.layers:
            x, st = layer.prefill(x)
            states.append(st)
        logits = self.lm_head(self.norm(x)[:, -1])
        out = [input_ids]
        for _ in range(max_new_tokens):
            nxt = _sample(logits, temperature, top_k)
            out.append(nxt)
            x = self.embedding(nxt.squeeze(1))
            for i, layer in enumerate(self.layers):
                x, states[i] = layer.step(x, states[i])
            logits = self.lm_head(self.norm(x))
        return torch.cat(out, dim=1)


def _sample(logits, temperature, top_k):
    """Sampling rule of the reference loop (mamba3/block.py:209-222)."""
    z = logits / temperature if temperature > 0 else logits
    if top_k is not None:
        v, _ = torch.topk(z, min(top_k, z.size(-1)))
        z = z.masked_fill(z < v[:, -1:], float("-inf"))
    if temperature > 0:
        return torch.multinomial(F.softmax(z, dim=-1), num_samples=1)
    return z.argmax(dim=-1, keepdim=True)
