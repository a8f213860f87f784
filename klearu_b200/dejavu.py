"""Deja Vu sparse FFN through the C ABI: the sparsity predictor and the
sparse SwiGLU MLP.

Mirrors klearu-dejavu's ``SparsityPredictor`` (predictor/mlp_predictor.rs:
``from_weights``, ``predict``, ``select_top_k``) and klearu-llm's
``sparse_mlp::forward_sparse`` (sparse/sparse_mlp.rs:4-37), batched over
tokens: inputs are ``[tokens][dim]`` and every call takes device tensors (or
anything ``torch.as_tensor`` accepts, moved to the context's GPU).
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import check
from .core import Context, default_context


def _host_f32(a, shape=None):
    a = np.ascontiguousarray(np.asarray(a, np.float32))
    if shape is not None and a.shape != shape:
        raise ValueError(f"expected shape {shape}, got {a.shape}")
    return a


def _dev(x, ctx: Context, dtype=torch.float32):
    return torch.as_tensor(x).to(device=f"cuda:{ctx.device}", dtype=dtype).contiguous()


class SparsityPredictor:
    """``SparsityPredictor::from_weights(w1, b1, w2, b2)``: w1 [hidden][input],
    w2 [output][hidden]; weights are held as bf16 on the GPU."""

    def __init__(self, w1, b1, w2, b2, ctx: Context | None = None):
        self.ctx = ctx or default_context()
        self.lib = self.ctx.lib
        w1 = _host_f32(w1)
        w2 = _host_f32(w2)
        self.hidden_dim, self.input_dim = w1.shape
        self.output_dim = w2.shape[0]
        b1 = _host_f32(b1, (self.hidden_dim,))
        b2 = _host_f32(b2, (self.output_dim,))
        _host_f32(w2, (self.output_dim, self.hidden_dim))
        h = C.c_void_p()
        check(self.lib.kl_predictor_create(self.ctx.h, self.input_dim, self.hidden_dim, self.output_dim,
                                           w1.ctypes.data, b1.ctypes.data, w2.ctypes.data, b2.ctypes.data,
                                           C.byref(h)), self.ctx.h, "kl_predictor_create")
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.kl_predictor_destroy(self.h)

    def predict(self, x) -> torch.Tensor:
        """Scores in [0, 1], [tokens][output_dim] (a 1-D input gives 1-D scores)."""
        xt = _dev(x, self.ctx)
        one = xt.dim() == 1
        xt = xt.reshape(-1, self.input_dim)
        out = torch.empty(xt.shape[0], self.output_dim, dtype=torch.float32, device=xt.device)
        check(self.lib.kl_predictor_predict(self.h, xt.data_ptr(), xt.shape[0], out.data_ptr()), self.ctx.h,
              "kl_predictor_predict")
        return out[0] if one else out

    def select_top_k(self, x, k: int) -> torch.Tensor:
        """Indices [tokens][min(k, output_dim)] (int64), highest score first,
        ties by lower index (the reference's stable sort)."""
        xt = _dev(x, self.ctx)
        one = xt.dim() == 1
        xt = xt.reshape(-1, self.input_dim)
        kk = min(int(k), self.output_dim)
        idx = torch.empty(xt.shape[0], kk, dtype=torch.int32, device=xt.device)
        check(self.lib.kl_predictor_select_topk(self.h, xt.data_ptr(), xt.shape[0], int(k), idx.data_ptr(), None),
              self.ctx.h, "kl_predictor_select_topk")
        idx = idx.long()
        return idx[0] if one else idx


class SparseMlp:
    """SwiGLU MLP weights: gate / up [intermediate][hidden], down
    [hidden][intermediate], optional down bias (klearu-dejavu mlp.rs)."""

    def __init__(self, gate, up, down, bias=None, ctx: Context | None = None):
        self.ctx = ctx or default_context()
        self.lib = self.ctx.lib
        gate = _host_f32(gate)
        self.intermediate_size, self.hidden_size = gate.shape
        up = _host_f32(up, gate.shape)
        down = _host_f32(down, (self.hidden_size, self.intermediate_size))
        b = None if bias is None else _host_f32(bias, (self.hidden_size,))
        h = C.c_void_p()
        check(self.lib.kl_sparse_mlp_create(self.ctx.h, self.hidden_size, self.intermediate_size, gate.ctypes.data,
                                            up.ctypes.data, down.ctypes.data, None if b is None else b.ctypes.data,
                                            C.byref(h)), self.ctx.h, "kl_sparse_mlp_create")
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.kl_sparse_mlp_destroy(self.h)

    def forward_sparse(self, x, selected) -> torch.Tensor:
        """``forward_sparse(x, active_neurons)`` per token: x [tokens][hidden],
        selected [tokens][k] neuron ids (summed in this order)."""
        xt = _dev(x, self.ctx)
        one = xt.dim() == 1
        xt = xt.reshape(-1, self.hidden_size)
        sel = _dev(selected, self.ctx, torch.int32).reshape(xt.shape[0], -1)
        out = torch.empty_like(xt)
        check(self.lib.kl_sparse_mlp_forward(self.h, xt.data_ptr(), xt.shape[0], sel.data_ptr(), sel.shape[1],
                                             out.data_ptr()), self.ctx.h, "kl_sparse_mlp_forward")
        return out[0] if one else out


class FfnStack:
    """The MLP half of klearu-llm's ``SparseModel::forward_decode_sparse``
    (sparse/mod.rs:112-141) over every layer: per layer RMSNorm, the layer's
    predictor top-k, the sparse SwiGLU MLP and the residual add, in one
    kl_ffn_stack_decode call (replayed as a CUDA graph for a repeated shape).
    ``predictors`` / ``mlps`` are lists of SparsityPredictor / SparseMlp on the
    same context; ``norm_weights`` is [layers][hidden]."""

    def __init__(self, predictors, mlps, norm_weights, eps: float = 1e-5, one_plus_weight: bool = False,
                 ctx: Context | None = None):
        self.ctx = ctx or default_context()
        self.lib = self.ctx.lib
        self._keep = (list(predictors), list(mlps))
        n = len(predictors)
        ph = (C.c_void_p * n)(*[p.h.value if hasattr(p.h, "value") else p.h for p in predictors])
        mh = (C.c_void_p * n)(*[m.h.value if hasattr(m.h, "value") else m.h for m in mlps])
        nw = _host_f32(norm_weights)
        self.hidden_size = nw.shape[1]
        h = C.c_void_p()
        check(self.lib.kl_ffn_stack_create(self.ctx.h, n, ph, mh, nw.ctypes.data, float(eps), int(one_plus_weight),
                                           C.byref(h)), self.ctx.h, "kl_ffn_stack_create")
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.kl_ffn_stack_destroy(self.h)

    def decode(self, hidden: torch.Tensor, neuron_sparsity: float) -> torch.Tensor:
        """Updates ``hidden`` [tokens][hidden] (a CUDA f32 tensor) in place and returns it."""
        assert hidden.is_cuda and hidden.dtype == torch.float32 and hidden.is_contiguous()
        check(self.lib.kl_ffn_stack_decode(self.h, hidden.data_ptr(), hidden.shape[0], float(neuron_sparsity)),
              self.ctx.h, "kl_ffn_stack_decode")
        return hidden
