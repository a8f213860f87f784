"""BOLT sparse inference over this library's LSH index
(crates/klearu-bolt/src/sparse_inference.rs: SparseInferenceEngine).

``SparseInferenceEngine(sparsity_multiplier).infer(input, index, weights,
biases, base_top_k)`` returns the [(neuron_id, activation)] list of the
reference: the index's candidates ordered by table count (descending; ties by
id ascending), the first int(base_top_k * multiplier) kept, activation =
ReLU(x . w + b) (``infer_linear``: no ReLU).  The batch forms run every input
in one kl_bolt_infer_batch call on the GPU; ``Network.bolt_infer`` uses a
trained network's layer.
"""

from __future__ import annotations


import numpy as np
import torch

from . import _lib
from ._lib import check
from .core import LshIndex, _ptr


class SparseInferenceEngine:
    def __init__(self, sparsity_multiplier: float):  # sparse_inference.rs:15-17
        self._mult = float(np.float32(sparsity_multiplier))

    def sparsity_multiplier(self) -> float:
        return self._mult

    def effective_k(self, base_top_k: int) -> int:  # sparse_inference.rs:40
        v = np.float32(base_top_k) * np.float32(self._mult)
        return 0 if not v > 0 else int(v)

    def infer_batch(self, X, index: LshIndex, weights, biases=None, base_top_k: int = 0, relu: bool = True,
                    stride: int | None = None):
        """Every row of X [n][d]: (ids [n][stride] uint32, activations [n][stride], counts [n])."""
        dev = index._dev
        X = torch.as_tensor(X).to(device=dev, dtype=torch.float32).contiguous()
        W = torch.as_tensor(weights).to(dev)
        dt = _lib.DTYPE_BF16 if W.dtype == torch.bfloat16 else _lib.DTYPE_F32
        W = (W if dt == _lib.DTYPE_BF16 else W.float()).contiguous()
        b = None if biases is None else torch.as_tensor(biases).to(device=dev, dtype=torch.float32).contiguous()
        n = X.shape[0]
        if stride is None:
            stride = max(1, min(self.effective_k(base_top_k), index.L * index.cap))
        ids = torch.zeros((n, stride), dtype=torch.int32, device=dev)
        act = torch.zeros((n, stride), dtype=torch.float32, device=dev)
        cnt = torch.zeros(n, dtype=torch.int32, device=dev)
        check(index.lib.kl_bolt_infer_batch(index.h, _ptr(W), dt, W.shape[1], _ptr(b), W.shape[0], _ptr(X), n,
                                            X.shape[1], self._mult, int(base_top_k), int(relu), _ptr(ids), _ptr(act),
                                            _ptr(cnt), stride), index.ctx.h, "kl_bolt_infer_batch")
        index.ctx.sync()
        return ids.cpu().numpy().view(np.uint32), act.cpu().numpy(), cnt.cpu().numpy()

    def infer(self, input, index: LshIndex, weights, biases=None, base_top_k: int = 0):  # sparse_inference.rs:32-70
        ids, act, cnt = self.infer_batch(np.asarray(input, np.float32)[None, :], index, weights, biases, base_top_k)
        return [(int(i), float(a)) for i, a in zip(ids[0, :cnt[0]], act[0, :cnt[0]])]

    def infer_linear(self, input, index: LshIndex, weights, biases=None, base_top_k: int = 0):  # :73-106
        ids, act, cnt = self.infer_batch(np.asarray(input, np.float32)[None, :], index, weights, biases, base_top_k,
                                         relu=False)
        return [(int(i), float(a)) for i, a in zip(ids[0, :cnt[0]], act[0, :cnt[0]])]


def network_bolt_infer(net, layer: int, X, sparsity_multiplier: float, base_top_k: int, relu: bool = True,
                       stride: int | None = None):
    """kl_net_bolt_infer: BOLT inference through layer `layer` (>= 1) of a
    trained Network; X is that layer's input."""
    dev = net._dev
    X = torch.as_tensor(X).to(device=dev, dtype=torch.float32).contiguous()
    n = X.shape[0]
    ix = net.layer_index(layer)
    eng = SparseInferenceEngine(sparsity_multiplier)
    if stride is None:
        stride = max(1, min(eng.effective_k(base_top_k), ix.L * ix.cap))
    ids = torch.zeros((n, stride), dtype=torch.int32, device=dev)
    act = torch.zeros((n, stride), dtype=torch.float32, device=dev)
    cnt = torch.zeros(n, dtype=torch.int32, device=dev)
    check(net.lib.kl_net_bolt_infer(net.h, layer, _ptr(X), n, X.shape[1], eng.sparsity_multiplier(), int(base_top_k),
                                    int(relu), _ptr(ids), _ptr(act), _ptr(cnt), stride), net.ctx.h,
          "kl_net_bolt_infer")
    net.ctx.sync()
    return ids.cpu().numpy().view(np.uint32), act.cpu().numpy(), cnt.cpu().numpy()
