"""Python mirror of CudaTransformer's ``FlashAttentionLayer<DType>``.

The reference declares the layer in ``cuda_transformer/FlashAttentionLayer.cu:13-150``:
public fields ``headDim, numHeads, cachedMaxScores, cachedDenominators,
cachedOutput, cachedBatchSize, cachedSequenceLength``, the constructor
``FlashAttentionLayer(headDim, numHeads)`` (:29), ``clone()`` (:34),
``computeAttention(q, k, v, saveStates=false)`` (:45-87),
``computeBackward(q, k, v, outputGrad)`` (:97-142) and ``clearCache()`` (:145).
This class keeps those names, argument meanings and ownership rules, with
torch CUDA tensors standing in for ``Tensor<DType>`` ([B, numHeads, T, headDim],
contiguous row-major).  Errors raise ``RuntimeError`` where the reference
throws ``std::runtime_error``.

Differences from the reference, all deliberate:
  * ``causal`` (constructor keyword, default False = the reference's
    behaviour) adds the causal mask the reference does not have.
  * The kernels keep an fp32 logsumexp per row (``cachedLSE``).  To stay
    consistent for code that reads the old cache fields,
    ``cachedMaxScores`` holds that logsumexp and ``cachedDenominators`` holds
    ones, so ``exp(s - max) / denom`` still gives the softmax.
  * dK and dV are the exact gradients (the reference kernel's are not,
    flash_attention.cu:310-321).
  * fp32: the forward rounds q, k, v to tf32 into a workspace; with saveStates
    that workspace is kept with the other cached state, and computeBackward
    reuses it (CTFA_DTYPE_TF32) when it is called on the same, unmodified
    q, k, v tensors.
"""
from __future__ import annotations

import torch

from . import _lib

_DTYPES = {
    torch.float32: _lib.CTFA_DTYPE_F32,
    torch.bfloat16: _lib.CTFA_DTYPE_BF16,
    torch.float16: _lib.CTFA_DTYPE_F16,
    torch.float64: _lib.CTFA_DTYPE_F64,
}


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class FlashAttentionLayer:
    """Flash attention core with cached forward state (not a ``Layer``;
    ``AttentionLayer`` owns one, ct/AttentionLayer.cu:15)."""

    def __init__(self, headDim: int, numHeads: int, causal: bool = False):
        self.headDim = int(headDim)
        self.numHeads = int(numHeads)
        self.causal = bool(causal)
        self.cachedMaxScores: torch.Tensor | None = None
        self.cachedDenominators: torch.Tensor | None = None
        self.cachedOutput: torch.Tensor | None = None
        self.cachedLSE: torch.Tensor | None = None
        self._cachedRounded = None  # (workspace, identity of q, k, v) for fp32
        self.cachedBatchSize = 0
        self.cachedSequenceLength = 0

    def clone(self) -> "FlashAttentionLayer":
        return FlashAttentionLayer(self.headDim, self.numHeads, self.causal)

    # -- helpers ---------------------------------------------------------
    def _check(self, *tensors: torch.Tensor) -> tuple[int, int, int]:
        q = tensors[0]
        if q.dim() != 4:
            raise RuntimeError(f"expected [batch, num_heads, seq_len, head_dim], got shape {tuple(q.shape)}")
        B, H, T, D = q.shape
        if H != self.numHeads or D != self.headDim:
            raise RuntimeError(
                f"tensor has {H} heads of dim {D}; layer was built for {self.numHeads} heads of dim {self.headDim}"
            )
        for t in tensors:
            if tuple(t.shape) != (B, H, T, D):
                raise RuntimeError(f"shape mismatch: {tuple(t.shape)} vs {(B, H, T, D)}")
            if t.dtype != q.dtype:
                raise RuntimeError("all tensors must share one dtype")
            if not t.is_cuda or t.device != q.device:
                raise RuntimeError("tensors must live on the same CUDA device")
            if not t.is_contiguous():
                raise RuntimeError("tensors must be contiguous (row-major [B, H, T, D])")
        if q.dtype not in _DTYPES:
            raise RuntimeError(f"unsupported dtype {q.dtype}")
        return B, T, _DTYPES[q.dtype]

    def _forward(self, lib, q, k, v, out, lse, B, T, dt):
        ws_bytes = lib.ctfa_forward_workspace_bytes(B, self.numHeads, T, self.headDim, dt)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
        with torch.cuda.device(q.device):
            status = lib.ctfa_forward(
                _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(lse), B, self.numHeads, T, self.headDim, dt,
                int(self.causal), _ptr(ws), ws_bytes, _stream_handle(q.device),
            )
            _lib.check(status, "ctfa_forward")
            if _lib.sync_check_enabled():
                _lib.check(lib.ctfa_check_device_error(_stream_handle(q.device)), "ctfa_forward (device)")
        return ws

    @staticmethod
    def _identity(*tensors):
        return tuple((t.data_ptr(), t._version) for t in tensors)

    # -- API -------------------------------------------------------------
    def computeAttention(
        self, queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, saveStates: bool = False
    ) -> torch.Tensor:
        B, T, dt = self._check(queries, keys, values)
        lib = _lib.load()
        output = torch.empty_like(queries)
        lse = torch.empty((B, self.numHeads, T), dtype=torch.float32, device=queries.device)
        ws = self._forward(lib, queries, keys, values, output, lse, B, T, dt)
        if saveStates:
            self._cachedRounded = (ws, self._identity(queries, keys, values)) if ws is not None else None
            self.cachedLSE = lse
            self.cachedMaxScores = lse.to(queries.dtype)
            self.cachedDenominators = torch.ones_like(self.cachedMaxScores)
            self.cachedOutput = output.clone()
            self.cachedBatchSize = B
            self.cachedSequenceLength = T
        return output

    def computeBackward(
        self, queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, outputGrad: torch.Tensor
    ) -> list[torch.Tensor]:
        B, T, dt = self._check(queries, keys, values, outputGrad)
        lib = _lib.load()
        output, lse = self.cachedOutput, self.cachedLSE
        if output is None or lse is None or self.cachedBatchSize != B or self.cachedSequenceLength != T:
            # Forward was not called with saveStates=True: recompute it
            # (FlashAttentionLayer.cu:114-127).
            output = torch.empty_like(queries)
            lse = torch.empty((B, self.numHeads, T), dtype=torch.float32, device=queries.device)
            self._forward(lib, queries, keys, values, output, lse, B, T, dt)
        dq = torch.empty_like(queries)
        dk = torch.empty_like(keys)
        dv = torch.empty_like(values)
        q_ptr, k_ptr, v_ptr = _ptr(queries), _ptr(keys), _ptr(values)
        cached = self._cachedRounded
        if cached is not None and cached[1] == self._identity(queries, keys, values):
            # the forward's tf32-rounded copies of these very tensors
            q_ptr, k_ptr, v_ptr = _lib.rounded_copies(cached[0], B, self.numHeads, T, self.headDim)
            dt = _lib.CTFA_DTYPE_TF32
        ws_bytes = lib.ctfa_backward_workspace_bytes(B, self.numHeads, T, self.headDim, dt)
        ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=queries.device)
        with torch.cuda.device(queries.device):
            status = lib.ctfa_backward(
                q_ptr, k_ptr, v_ptr, _ptr(output), _ptr(outputGrad), _ptr(lse),
                _ptr(dq), _ptr(dk), _ptr(dv), _ptr(ws), ws.numel(),
                B, self.numHeads, T, self.headDim, dt, int(self.causal), _stream_handle(queries.device),
            )
            _lib.check(status, "ctfa_backward")
            if _lib.sync_check_enabled():
                _lib.check(lib.ctfa_check_device_error(_stream_handle(queries.device)), "ctfa_backward (device)")
        return [dq, dk, dv]

    def clearCache(self) -> None:
        self.cachedMaxScores = None
        self.cachedDenominators = None
        self.cachedOutput = None
        self.cachedLSE = None
        self._cachedRounded = None
