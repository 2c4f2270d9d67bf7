"""Token-by-token decode of a KulaMambaLM with one CUDA graph per decode step.

KulaMambaLM.generate (mamba3/block.py:195-231) pays a Python round trip and a launch per
operation for every layer of every token.  GraphDecoder keeps every layer's inference state
in static fp32 buffers, updates them in place with the step kernel, and captures one whole
decode step -- embedding, the layers (norms, in_proj, step kernel, out_proj, MLP), final
norm, lm_head and the sampling rule -- in a CUDA graph that it replays once per token.  The
tokens collect on the device; the host reads them once at the end.

Same results as KulaMambaLM.generate with the same sampling arguments; greedy decoding
(temperature 0) is deterministic.  The sampling rule is part of the captured step, so the
decoder keeps one graph per (temperature, top_k) that prefill() has been given.  By default
the decoder keeps each layer's previous token in the compact form (its rotated B^ and MIMO x,
allocate_inference_state(compact=True)), which halves the state bytes every step moves;
compact=False keeps the reference's prev_BX.
"""

from __future__ import annotations

import torch

from . import ops
from .block import _residual


class GraphDecoder:
    def __init__(self, lm, batch_size: int, max_new_tokens: int, compact: bool = True):
        self.lm = lm
        self.B = int(batch_size)
        self.n = int(max_new_tokens)
        p = next(lm.parameters())
        self.dev = p.device
        if self.dev.type != "cuda":
            raise RuntimeError("GraphDecoder needs the model on a CUDA device")
        self.layers = list(lm.layers)
        self.compact = bool(compact)
        self.states = [blk.ssm.allocate_inference_state(self.B, device=self.dev, compact=self.compact)
                       for blk in self.layers]
        self.dims = [self._dims(blk.ssm) for blk in self.layers]
        self.ybuf = [torch.empty(self.B, blk.ssm.nheads * blk.ssm.headdim, dtype=p.dtype, device=self.dev)
                     for blk in self.layers]
        self.tok = torch.zeros(self.B, 1, dtype=torch.long, device=self.dev)
        self.out = torch.zeros(self.B, max(1, self.n), dtype=torch.long, device=self.dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=self.dev)
        self.graphs = {}  # one captured step per sampling rule (temperature, top_k)
        self.step_ws = None
        self.sampling = None

    @staticmethod
    def _dims(ssm):
        d = ssm._dims()
        return (d["H"], d["P"], d["N"], d["R"], d["G"], d["trapezoidal"], d["complex_ssm"], d["norm_eps"])

    def _add_norm(self, x, h, scale, norm):
        """(x + h * scale, norm of it): one kernel for 16-bit activations, else the two the eager
        path runs (both store the same values)."""
        if x.dtype in (torch.bfloat16, torch.float16) and x.shape[-1] % 8 == 0:
            return ops.add_rmsnorm(x, h, scale, norm.weight, norm.eps)
        x = _residual(x, h, scale)
        return x, norm(x)

    def _layer_step(self, i, blk, x, n):
        """Block i on the residual stream x with n = its ssm_norm(x); returns the stream after the
        block and the next norm (the next block's ssm_norm, or the LM's final norm) of it, each
        residual add fused with the norm that follows it."""
        ssm = blk.ssm
        proj = ssm.in_proj(n)
        st = self.states[i]
        # one step workspace for every layer (the layers run one after another on one stream);
        # allocated by the first, uncaptured step
        if self.compact:
            self.step_ws = ops.step_ssm_compact_(ssm._param_tensors(), self.dims[i], proj, st["h"], st["prev_B"],
                                                 st["prev_x"], st["angle"], self.ybuf[i], workspace=self.step_ws)
        else:
            self.step_ws = ops.step_ssm_(ssm._param_tensors(), self.dims[i], proj, st["h"], st["prev_BX"],
                                         st["angle"], self.ybuf[i], workspace=self.step_ws)
        h = ssm.out_proj(self.ybuf[i])
        nxt = self.layers[i + 1].ssm_norm if i + 1 < len(self.layers) else self.lm.norm
        if blk.use_mlp:
            x, n1 = self._add_norm(x, h, blk.residual_scale, blk.mlp_norm)
            return self._add_norm(x, blk.mlp(n1), blk.residual_scale, nxt)
        return self._add_norm(x, h, blk.residual_scale, nxt)

    def _sample(self, logits):
        from .block import _sample

        temperature, top_k = self.sampling
        return _sample(logits, temperature, top_k)

    def _decode_body(self):
        """One token: self.tok -> layers -> next token in self.tok and in self.out[:, pos]."""
        x = self.lm.embedding(self.tok.squeeze(1))
        n = self.layers[0].ssm_norm(x)
        for i, blk in enumerate(self.layers):
            x, n = self._layer_step(i, blk, x, n)
        logits = self.lm.lm_head(n)
        nxt = self._sample(logits)
        self.tok.copy_(nxt)
        self.out.scatter_(1, self.pos.view(1, 1).expand(self.B, 1), nxt)
        self.pos.add_(1)

    @torch.no_grad()
    def prefill(self, input_ids, temperature=0.0, top_k=None):
        """Run every layer's prefill on the prompt, load the static states and pick the first token."""
        if input_ids.shape[0] != self.B:
            raise ValueError(f"batch {input_ids.shape[0]} != decoder batch {self.B}")
        self.sampling = (float(temperature), top_k)
        x = self.lm.embedding(input_ids)
        for i, blk in enumerate(self.layers):
            x, st = blk.prefill(x, compact_state=self.compact)
            for k in self.states[i]:
                self.states[i][k].copy_(st[k])
        logits = self.lm.lm_head(self.lm.norm(x)[:, -1])
        self.tok.copy_(self._sample(logits))
        self.pos.zero_()

    def _capture(self):
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        saved = [{k: v.clone() for k, v in st.items()} for st in self.states]
        tok0, pos0 = self.tok.clone(), self.pos.clone()
        with torch.cuda.stream(s):  # warm the allocator and cuBLAS outside the capture
            self._decode_body()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self._decode_body()
        # the warm-up step advanced the state: restore it
        for st, sv in zip(self.states, saved):
            for k in st:
                st[k].copy_(sv[k])
        self.tok.copy_(tok0)
        self.pos.copy_(pos0)
        self.graphs[self.sampling] = g

    @torch.no_grad()
    def decode(self, steps=None):
        """Replay the captured step `steps` times (default max_new_tokens); tokens stay on device."""
        steps = self.n if steps is None else int(steps)
        if steps > self.n:
            raise ValueError("more steps than max_new_tokens")
        if self.sampling is None:
            raise RuntimeError("decode() before prefill()")
        if self.sampling not in self.graphs:  # the sampling rule is baked into the captured step
            self._capture()
        g = self.graphs[self.sampling]
        first = self.tok.clone()
        for _ in range(steps):
            g.replay()
        return first, self.out[:, :steps]

    @torch.no_grad()
    def generate(self, input_ids, temperature=0.0, top_k=None):
        """Same contract as KulaMambaLM.generate: the prompt followed by max_new_tokens tokens."""
        self.prefill(input_ids, temperature, top_k)
        first, rest = self.decode(max(0, self.n - 1))
        return torch.cat([input_ids, first, rest], dim=1)
