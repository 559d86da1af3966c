"""Python mirrors of CudaTransformer's ``QKVProjectionLayer<DType>`` and
``OutputProjectionLayer<DType>``, the two steps either side of the attention
core in ``AttentionLayer``, over the projection entry points of
libctfa_b200.so (tcgen05 GEMMs that read and write the head layout
``[B, H, T, D]`` directly).

Reference API kept (names, argument meaning, shapes, ownership):

* ``QKVProjectionLayer(inputDim, numHeads, headDim)``
  (``cuda_transformer/QKVProjectionLayer.cu:13-144``): fields
  ``weights{Query,Key,Value}``, ``biases{Query,Key,Value}`` and their
  ``...Grad`` twins (gradients allocated zero-filled by the first backward,
  :107-116), ``clone()`` (:52), ``computeQKV(input)`` -> ``[q, k, v]``
  (:73-96), ``computeBackward(input, queryGrad, keyGrad, valueGrad)`` ->
  ``inputGrad`` (:100-141; parameter gradients ACCUMULATE across calls, as the
  reference's atomicAdd kernels do).
* ``OutputProjectionLayer(inputDim, headDim, numHeads)``
  (``cuda_transformer/OutputProjectionLayer.cu:11-100``): fields
  ``weightsProj``, ``biasesProj``, ``weightsProjGrad``, ``biasesProjGrad``,
  ``clone()`` (:40), ``forward(input)`` (:52-66), ``backward(input,
  gradOutput)`` (:69-97).

Weights are held as the reference's kernels index the buffers: the QKV
weights as ``[numHeads*headDim, inputDim]`` (row = output feature,
attention_qkv_kernels.cu:92) and the output weights as
``[inputDim, numHeads*headDim]`` (attention_proj_kernels.cu:83).  The
reference allocates them zero-filled (headers.cu:196-214); so do these
classes.  Torch CUDA tensors stand in for ``Tensor<DType>``.
"""
from __future__ import annotations

import torch

from . import _lib
from .flash_attention_layer import _DTYPES, _stream_handle


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _code(t: torch.Tensor) -> int:
    if t.dtype not in _DTYPES:
        raise RuntimeError(f"unsupported dtype {t.dtype}")
    if not t.is_cuda:
        raise RuntimeError("projection tensors must live on a CUDA device")
    return _DTYPES[t.dtype]


def _contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------------------
# Functional wrappers of the C ABI (no autograd)
# ---------------------------------------------------------------------------
def qkv_forward(x, wq, bq, wk, bk, wv, bv, num_heads: int, head_dim: int):
    """q, k, v [B, H, T, D] = x [.., T, E] W^T + b (ctfa_qkv_forward)."""
    x = _contig(x)
    T, E = x.shape[-2], x.shape[-1]
    B = x.numel() // (T * E)
    out = [torch.empty(B, num_heads, T, head_dim, dtype=x.dtype, device=x.device) for _ in range(3)]
    lib = _lib.load()
    _lib.check(
        lib.ctfa_qkv_forward(_p(x), _p(_contig(wq)), _p(bq), _p(_contig(wk)), _p(bk), _p(_contig(wv)), _p(bv),
                             _p(out[0]), _p(out[1]), _p(out[2]), B, T, E, num_heads, head_dim, _code(x),
                             _stream_handle(x.device)),
        "ctfa_qkv_forward",
    )
    return out


def qkv_backward(x, dq, dk, dv, wq, wk, wv, dwq=None, dbq=None, dwk=None, dbk=None, dwv=None, dbv=None,
                 want_dx: bool = True):
    """dx [B, T, E] (or None) and, when given, dW/db ADDED into dwq.. / dbq..
    (ctfa_qkv_backward)."""
    dq, dk, dv = _contig(dq), _contig(dk), _contig(dv)
    B, H, T, D = dq.shape
    E = wq.shape[-1] if wq is not None else x.shape[-1]
    dx = torch.empty(B, T, E, dtype=dq.dtype, device=dq.device) if want_dx else None
    lib = _lib.load()
    _lib.check(
        lib.ctfa_qkv_backward(_p(x if x is None else _contig(x)), _p(dq), _p(dk), _p(dv), _p(wq), _p(wk), _p(wv),
                              _p(dwq), _p(dbq), _p(dwk), _p(dbk), _p(dwv), _p(dbv), _p(dx), B, T, E, H, D,
                              _code(dq), _stream_handle(dq.device)),
        "ctfa_qkv_backward",
    )
    return dx


def out_proj_forward(a, wo, bo):
    """y [B, T, E] = a (heads concatenated per row) Wo^T + bo (ctfa_out_proj_forward)."""
    a = _contig(a)
    B, H, T, D = a.shape
    E = wo.shape[0]
    y = torch.empty(B, T, E, dtype=a.dtype, device=a.device)
    lib = _lib.load()
    _lib.check(
        lib.ctfa_out_proj_forward(_p(a), _p(_contig(wo)), _p(bo), _p(y), B, T, E, H, D, _code(a),
                                  _stream_handle(a.device)),
        "ctfa_out_proj_forward",
    )
    return y


def out_proj_backward(a, dy, wo, dwo=None, dbo=None, want_da: bool = True, num_heads: int | None = None,
                      head_dim: int | None = None):
    """da [B, H, T, D] (or None) and, when given, dWo / dbo ADDED
    (ctfa_out_proj_backward)."""
    dy = _contig(dy)
    if a is not None:
        B, H, T, D = a.shape
    else:
        H, D = num_heads, head_dim
        T, E_ = dy.shape[-2], dy.shape[-1]
        B = dy.numel() // (T * E_)
    E = dy.shape[-1]
    da = torch.empty(B, H, T, D, dtype=dy.dtype, device=dy.device) if want_da else None
    lib = _lib.load()
    _lib.check(
        lib.ctfa_out_proj_backward(_p(a if a is None else _contig(a)), _p(dy), _p(wo), _p(dwo), _p(dbo), _p(da),
                                   B, T, E, H, D, _code(dy), _stream_handle(dy.device)),
        "ctfa_out_proj_backward",
    )
    return da


# ---------------------------------------------------------------------------
# Layer mirrors
# ---------------------------------------------------------------------------
class QKVProjectionLayer:
    """Projects [batch, seq_len, inputDim] input to multi-head q, k, v."""

    def __init__(self, inputDim: int, numHeads: int, headDim: int, dtype: torch.dtype = torch.float32,
                 device: torch.device | str | None = None):
        self.inputDim, self.numHeads, self.headDim = int(inputDim), int(numHeads), int(headDim)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        hd = self.numHeads * self.headDim
        zeros = lambda *s: torch.zeros(*s, dtype=dtype, device=dev)
        self.weightsQuery, self.weightsKey, self.weightsValue = zeros(hd, inputDim), zeros(hd, inputDim), zeros(hd, inputDim)
        self.biasesQuery, self.biasesKey, self.biasesValue = zeros(hd), zeros(hd), zeros(hd)
        self.weightsQueryGrad = self.weightsKeyGrad = self.weightsValueGrad = None
        self.biasesQueryGrad = self.biasesKeyGrad = self.biasesValueGrad = None

    def clone(self) -> "QKVProjectionLayer":
        c = QKVProjectionLayer(self.inputDim, self.numHeads, self.headDim, self.weightsQuery.dtype,
                               self.weightsQuery.device)
        for n in ("weightsQuery", "weightsKey", "weightsValue", "biasesQuery", "biasesKey", "biasesValue"):
            getattr(c, n).copy_(getattr(self, n))
        return c

    def computeQKV(self, input: torch.Tensor) -> list[torch.Tensor]:
        if input.shape[-1] != self.inputDim:
            raise RuntimeError(f"input feature size {input.shape[-1]} != inputDim {self.inputDim}")
        return qkv_forward(input, self.weightsQuery, self.biasesQuery, self.weightsKey, self.biasesKey,
                           self.weightsValue, self.biasesValue, self.numHeads, self.headDim)

    def computeBackward(self, input, queryGrad, keyGrad, valueGrad) -> torch.Tensor:
        if self.weightsQueryGrad is None:
            z = lambda t: torch.zeros_like(t)
            self.weightsQueryGrad, self.weightsKeyGrad, self.weightsValueGrad = (
                z(self.weightsQuery), z(self.weightsKey), z(self.weightsValue))
            self.biasesQueryGrad, self.biasesKeyGrad, self.biasesValueGrad = (
                z(self.biasesQuery), z(self.biasesKey), z(self.biasesValue))
        dx = qkv_backward(input, queryGrad, keyGrad, valueGrad, self.weightsQuery, self.weightsKey,
                          self.weightsValue, self.weightsQueryGrad, self.biasesQueryGrad, self.weightsKeyGrad,
                          self.biasesKeyGrad, self.weightsValueGrad, self.biasesValueGrad)
        return dx.view(input.shape)


class OutputProjectionLayer:
    """Projects the concatenated heads [B, H, T, D] back to inputDim."""

    def __init__(self, inputDim: int, headDim: int, numHeads: int, dtype: torch.dtype = torch.float32,
                 device: torch.device | str | None = None):
        self.inputDim, self.headDim, self.numHeads = int(inputDim), int(headDim), int(numHeads)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.weightsProj = torch.zeros(inputDim, numHeads * headDim, dtype=dtype, device=dev)
        self.biasesProj = torch.zeros(inputDim, dtype=dtype, device=dev)
        self.weightsProjGrad = None
        self.biasesProjGrad = None

    def clone(self) -> "OutputProjectionLayer":
        c = OutputProjectionLayer(self.inputDim, self.headDim, self.numHeads, self.weightsProj.dtype,
                                  self.weightsProj.device)
        c.weightsProj.copy_(self.weightsProj)
        c.biasesProj.copy_(self.biasesProj)
        return c

    def _heads(self, input: torch.Tensor) -> torch.Tensor:
        if input.dim() != 4 or input.shape[1] != self.numHeads or input.shape[3] != self.headDim:
            raise RuntimeError(f"expected [batch, {self.numHeads}, seq_len, {self.headDim}], got {tuple(input.shape)}")
        return input

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        return out_proj_forward(self._heads(input), self.weightsProj, self.biasesProj)

    def backward(self, input: torch.Tensor, gradOutput: torch.Tensor) -> torch.Tensor:
        if self.weightsProjGrad is None:
            self.weightsProjGrad = torch.zeros_like(self.weightsProj)
            self.biasesProjGrad = torch.zeros_like(self.biasesProj)
        return out_proj_backward(self._heads(input), gradOutput, self.weightsProj, self.weightsProjGrad,
                                 self.biasesProjGrad)
