"""LLaMA MLP modules backed by the B200 kernels.

``SvdLlamaMLP`` is the B200 counterpart of the reference's
``NeuronLlamaMLP_SVD`` (models/modeling_llama.py:796-893): it holds the six
factors (reference names: ``u_*`` first factor [in, r], ``v_*`` second factor
[r, out]), packs them once, and its ``forward`` reshapes ``[B, S, H]`` to
``[B*S, H]``, runs the fused SVD layer and reshapes back
(``_kernel_enabled_mlp``, models/modeling_llama.py:840-863).
``from_torch_linear_factors`` accepts the checkpoint's PyTorch ``[out, in]``
order (``gate_v_proj`` = first factor, models/modeling_llama.py:1105-1113).

``MlpBlockStack`` is the MLP-only decoder stack of the benchmark
configurations (bench/e2e_block.py:264-278 without attention): per layer
``x = x + mlp(rmsnorm(x))``, with the residual add fused into the last GEMM's
epilogue; it can be captured into one CUDA graph.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from ..kernels import ops


class SvdLlamaMLP(torch.nn.Module):
    def __init__(self, u_gate, v_gate, u_up, v_up, u_down, v_down, *, mlp_kernel_enabled: bool = True):
        super().__init__()
        if not mlp_kernel_enabled:
            raise NotImplementedError("the B200 module always runs the fused kernels (no XLA/eager path)")
        self.hidden_size = u_gate.shape[0]
        self.intermediate_size = v_gate.shape[1]
        self.rank = u_gate.shape[1]
        self.layer = ops.pack_svd_layer(u_gate, v_gate, u_up, v_up, u_down, v_down)

    @classmethod
    def from_torch_linear_factors(cls, gate_v_proj, gate_u_proj, up_v_proj, up_u_proj, down_v_proj, down_u_proj):
        """Factors in torch.nn.Linear order ([out, in]): *_v_proj [r, in], *_u_proj [out, r]."""
        return cls(gate_v_proj.t(), gate_u_proj.t(), up_v_proj.t(), up_u_proj.t(), down_v_proj.t(), down_u_proj.t())

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        r2 = None if residual is None else residual.reshape(-1, shape[-1])
        y = ops.svd_mlp_packed(self.layer, x2, residual=r2)
        if x.dtype != torch.bfloat16:
            y = y.to(x.dtype)
        return y.reshape(*shape[:-1], self.hidden_size)


class DenseLlamaMLP(torch.nn.Module):
    """Dense SwiGLU MLP (models/modeling_llama.py:900-943) on the same kernels."""

    def __init__(self, w_gate, w_up, w_down):
        super().__init__()
        self.hidden_size = w_gate.shape[0]
        self.layer = ops.pack_dense_layer(w_gate, w_up, w_down)

    @classmethod
    def from_torch_linear(cls, gate_proj, up_proj, down_proj):
        """Weights in torch.nn.Linear order: gate/up [I, H], down [H, I]."""
        return cls(gate_proj.t(), up_proj.t(), down_proj.t())

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        r2 = None if residual is None else residual.reshape(-1, shape[-1])
        y = ops.dense_mlp_packed(self.layer, x2, residual=r2)
        if x.dtype != torch.bfloat16:
            y = y.to(x.dtype)
        return y.reshape(*shape[:-1], self.hidden_size)


class MlpBlockStack:
    """N blocks of x = x + mlp(rmsnorm(x)) (RMSNorm eps 1e-5 by default)."""

    def __init__(self, mlps: Sequence[torch.nn.Module], norm_weights: Sequence[torch.Tensor], eps: float = 1e-5):
        if len(mlps) != len(norm_weights):
            raise ValueError("one norm weight per layer")
        self.mlps = list(mlps)
        self.norms = [w.to(torch.bfloat16).contiguous() for w in norm_weights]
        self.eps = eps
        self._graph = None
        self._static_in = None
        self._static_out = None

    def _run(self, x: torch.Tensor, buf_a: torch.Tensor, buf_b: torch.Tensor, normed: torch.Tensor) -> torch.Tensor:
        cur = x
        outs = (buf_a, buf_b)
        for i, (mlp, w) in enumerate(zip(self.mlps, self.norms)):
            ops.rmsnorm(cur, w, self.eps, out=normed)
            nxt = outs[i % 2]
            if isinstance(mlp, SvdLlamaMLP):
                ops.svd_mlp_packed(mlp.layer, normed, residual=cur, out=nxt)
            else:
                ops.dense_mlp_packed(mlp.layer, normed, residual=cur, out=nxt)
            cur = nxt
        return cur

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x: [M, H] bf16 -> [M, H] bf16 (eager launches)."""
        x = x.to(torch.bfloat16).contiguous()
        a, b, n = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
        return self._run(x, a, b, n).clone()

    __call__ = forward

    def capture(self, m: int, hidden: int, device) -> None:
        """Captures the whole stack for M tokens into one CUDA graph."""
        self._static_in = torch.zeros((m, hidden), dtype=torch.bfloat16, device=device)
        a, b, n = (torch.empty_like(self._static_in) for _ in range(3))
        self._bufs = (a, b, n)
        # warm up outside capture: workspaces are allocated on first use
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            self._run(self._static_in, a, b, n)
        torch.cuda.current_stream(device).wait_stream(s)
        torch.cuda.synchronize(device)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph, stream=s):
            self._static_out = self._run(self._static_in, a, b, n)

    def replay(self, x: torch.Tensor) -> torch.Tensor:
        if self._graph is None:
            raise RuntimeError("call capture() first")
        self._static_in.copy_(x)
        self._graph.replay()
        return self._static_out
