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
epilogue; it can be captured into one CUDA graph.  ``SvdMlpBlock`` is one such
block with the RMSNorm fused as well (the norm weight folded into u_gate/u_up,
the per-row statistics written by the previous block's residual epilogue); a
stack of them launches no norm kernel except one statistics pass at its input.
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


class SvdMlpBlock(torch.nn.Module):
    """x + SvdLlamaMLP(rmsnorm(x) * norm_weight) with the norm fused into the
    layer (svdmlp_forward_block); RMSNorm as LlamaRMSNorm
    (models/modeling_llama.py:1140-1152 applies it before the MLP)."""

    def __init__(self, u_gate, v_gate, u_up, v_up, u_down, v_down, norm_weight, eps: float = 1e-5):
        super().__init__()
        self.hidden_size = u_gate.shape[0]
        self.intermediate_size = v_gate.shape[1]
        self.rank = u_gate.shape[1]
        self.eps = float(eps)
        self.layer = ops.pack_svd_layer(u_gate, v_gate, u_up, v_up, u_down, v_down, norm_weight=norm_weight)

    def block(self, x: torch.Tensor, x_stats: torch.Tensor, y_stats: Optional[torch.Tensor] = None,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """[M, H] bf16 with its row statistics (ops.row_sumsq) -> [M, H] bf16."""
        return ops.svd_block_packed(self.layer, x, x_stats, y_stats=y_stats, eps=self.eps, out=out)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        y = self.block(x2, ops.row_sumsq(x2))
        if x.dtype != torch.bfloat16:
            y = y.to(x.dtype)
        return y.reshape(shape)


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
    """N blocks of x = x + mlp(rmsnorm(x)) (RMSNorm eps 1e-5 by default).

    Blocks given as SvdMlpBlock carry their own norm (their entry of
    `norm_weights` may be None) and run fused: each one's residual epilogue
    writes the statistics the next one normalises with."""

    def __init__(self, mlps: Sequence[torch.nn.Module], norm_weights: Optional[Sequence[torch.Tensor]] = None,
                 eps: float = 1e-5):
        self.mlps = list(mlps)
        if norm_weights is None:
            norm_weights = [None] * len(self.mlps)
        if len(self.mlps) != len(norm_weights):
            raise ValueError("one norm weight per layer")
        self.norms = []
        for mlp, w in zip(self.mlps, norm_weights):
            if isinstance(mlp, SvdMlpBlock):
                self.norms.append(None)
            elif w is None:
                raise ValueError("a layer that is not an SvdMlpBlock needs its norm weight")
            else:
                self.norms.append(w.to(torch.bfloat16).contiguous())
        self.eps = eps
        self._graph = None
        self._static_in = None
        self._static_out = None

    def _stats_shape(self, x: torch.Tensor):
        return (2, x.shape[0], -(-x.shape[1] // 128))

    def _run(self, x: torch.Tensor, buf_a: torch.Tensor, buf_b: torch.Tensor, normed: torch.Tensor,
             stats: Optional[torch.Tensor] = None) -> torch.Tensor:
        cur = x
        outs = (buf_a, buf_b)
        have_stats = None            # index of the stats buffer that holds cur's statistics
        n = len(self.mlps)
        for i, (mlp, w) in enumerate(zip(self.mlps, self.norms)):
            nxt = outs[i % 2]
            if isinstance(mlp, SvdMlpBlock):
                if have_stats is None:
                    have_stats = 0
                    ops.row_sumsq(cur, out=stats[0])
                nxt_fused = i + 1 < n and isinstance(self.mlps[i + 1], SvdMlpBlock)
                y_stats = stats[1 - have_stats] if nxt_fused else None
                mlp.block(cur, stats[have_stats], y_stats=y_stats, out=nxt)
                have_stats = 1 - have_stats if nxt_fused else None
            else:
                ops.rmsnorm(cur, w, self.eps, out=normed)
                if isinstance(mlp, SvdLlamaMLP):
                    ops.svd_mlp_packed(mlp.layer, normed, residual=cur, out=nxt)
                else:
                    ops.dense_mlp_packed(mlp.layer, normed, residual=cur, out=nxt)
                have_stats = None
            cur = nxt
        return cur

    def _buffers(self, x: torch.Tensor):
        a, b, n = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
        stats = torch.empty(self._stats_shape(x), dtype=torch.float32, device=x.device)
        return a, b, n, stats

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x: [M, H] bf16 -> [M, H] bf16 (eager launches)."""
        x = x.to(torch.bfloat16).contiguous()
        return self._run(x, *self._buffers(x)).clone()

    __call__ = forward

    def capture(self, m: int, hidden: int, device) -> None:
        """Captures the whole stack for M tokens into one CUDA graph."""
        self._static_in = torch.zeros((m, hidden), dtype=torch.bfloat16, device=device)
        a, b, n, stats = self._buffers(self._static_in)
        self._bufs = (a, b, n, stats)
        # warm up outside capture: workspaces are allocated on first use
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            self._run(self._static_in, a, b, n, stats)
        torch.cuda.current_stream(device).wait_stream(s)
        torch.cuda.synchronize(device)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph, stream=s):
            self._static_out = self._run(self._static_in, a, b, n, stats)

    def replay(self, x: torch.Tensor) -> torch.Tensor:
        if self._graph is None:
            raise RuntimeError("call capture() first")
        self._static_in.copy_(x)
        self._graph.replay()
        return self._static_out
