"""PyTorch-facing wrappers of the C-ABI entry points.

Tensors stay owned by PyTorch; the library only receives raw pointers and the
current CUDA stream (the reference launches on the engine stream,
``model_executor/engine.py:50-51``). Nothing here falls back to PyTorch math.
"""

from __future__ import annotations

import ctypes
import threading
from typing import Dict, Optional, Tuple

import torch

from ._lib import c_i64, call, check, lib

DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1}


def _p(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


try:  # the raw handle without building a Stream object (~0.2 us instead of ~2 us)
    _raw_stream = torch._C._cuda_getCurrentRawStream
    _cur_device = torch._C._cuda_getDevice
except AttributeError:  # pragma: no cover - older torch
    def _raw_stream(idx: int) -> int:
        return torch.cuda.current_stream(idx).cuda_stream

    _cur_device = torch.cuda.current_device


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype not in DTYPE_CODE:
        raise ValueError(f"activation dtype {dtype} not supported (float16 or bfloat16)")
    return DTYPE_CODE[dtype]


class _DeviceGuard:
    """Makes ``device`` current for the library's CUDA runtime calls."""

    def __init__(self, device: torch.device):
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def _check_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError("tensors must live on a CUDA device (there is no CPU path)")
        if t.device != dev:
            raise ValueError("tensors must live on the same device")
        if not t.is_contiguous():
            raise ValueError("tensors must be contiguous")
    return dev


# ---------------------------------------------------------------- repack
def blob_bytes(K: int, N: int, G: int) -> int:
    out = c_i64(0)
    call("awqb_blob_bytes", K, N, G, ctypes.byref(out))
    return out.value


def repack(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, group_size: int) -> torch.Tensor:
    """AWQ (qweight [.., K, N/8], qzeros, scales) -> blob (uint8 [.., bytes])."""
    batched = qweight.dim() == 3
    qw = qweight if batched else qweight.unsqueeze(0)
    qz = qzeros if batched else qzeros.unsqueeze(0)
    sc = scales if batched else scales.unsqueeze(0)
    E, K, N8 = qw.shape
    N = N8 * 8
    G = K if group_size == -1 else group_size
    if qw.dtype != torch.int32 or qz.dtype != torch.int32:
        raise ValueError("qweight and qzeros must be int32")
    if sc.dtype not in DTYPE_CODE:
        raise ValueError("scales must be float16 or bfloat16")
    if qz.shape != (E, K // G, N8) or sc.shape != (E, K // G, N):
        raise ValueError(f"inconsistent AWQ shapes {tuple(qw.shape)} {tuple(qz.shape)} {tuple(sc.shape)}")
    dev = _check_cuda(qw, qz, sc)
    nb = blob_bytes(K, N, G)
    blob = torch.empty((E, nb), dtype=torch.uint8, device=dev)
    with _DeviceGuard(dev):
        call("awqb_repack", _p(qw), _p(qz), _p(sc), E, K, N, G, _p(blob), _stream(dev))
    return blob if batched else blob[0]


def unrepack(blob: torch.Tensor, K: int, N: int, G: int, scale_dtype: torch.dtype
             ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    batched = blob.dim() == 2
    b = blob if batched else blob.unsqueeze(0)
    E = b.shape[0]
    dev = _check_cuda(b)
    qw = torch.empty((E, K, N // 8), dtype=torch.int32, device=dev)
    qz = torch.empty((E, K // G, N // 8), dtype=torch.int32, device=dev)
    sc = torch.empty((E, K // G, N), dtype=scale_dtype, device=dev)
    with _DeviceGuard(dev):
        call("awqb_unrepack", _p(b), E, K, N, G, _p(qw), _p(qz), _p(sc), _stream(dev))
    if not batched:
        return qw[0], qz[0], sc[0]
    return qw, qz, sc


def dequant(blob: torch.Tensor, K: int, N: int, G: int, dtype: torch.dtype) -> torch.Tensor:
    """W = (q - z) * s in ``dtype``: [.., K, N]."""
    batched = blob.dim() == 2
    b = blob if batched else blob.unsqueeze(0)
    E = b.shape[0]
    dev = _check_cuda(b)
    w = torch.empty((E, K, N), dtype=dtype, device=dev)
    with _DeviceGuard(dev):
        call("awqb_dequant", _p(b), E, K, N, G, _dtype_code(dtype), _p(w), _stream(dev))
    return w if batched else w[0]


# ---------------------------------------------------------------- workspace
class _WorkspacePool:
    """One zero-filled scratch buffer per device, grown on demand.

    The GEMM keeps its split-tile counters in the first 8 KiB of any workspace
    and leaves them at zero after every call that completes, so the buffer is
    zeroed only when it is (re)allocated; the rest is scratch shared by calls of
    every shape. A call whose bounded device wait gave up (``device_error``
    non-zero) can leave counters set: ``clear_device_error`` zeroes the counter
    region of every pool buffer together with the error word.

    One buffer serves every stream of a device, so pool-backed calls must not
    run concurrently on different streams (they would share counters and
    partial tiles); pass ``workspace=`` to give concurrent streams their own.
    Growing is refused while a CUDA graph is being captured: size it first
    (``reserve``) with the largest call.
    """

    def __init__(self):
        self._bufs: Dict[int, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        buf = self._bufs.get(idx)
        if buf is not None and buf.numel() >= nbytes:
            return buf
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("AWQ GEMM workspace must be reserved before CUDA graph capture")
        with self._lock:
            buf = self._bufs.get(idx)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 20)
                if buf is not None:
                    size = max(size, 2 * buf.numel())
                buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
                self._bufs[idx] = buf
        return buf

    def reserve(self, device: torch.device, nbytes: int) -> None:
        self.get(device, nbytes)

    def reset_counters(self) -> None:
        """Zero the split-tile counter region of every buffer (on each
        device's current stream)."""
        with self._lock:
            for idx, buf in self._bufs.items():
                with torch.cuda.device(idx):
                    buf[:COUNTER_BYTES].zero_()


# Split-tile counters at the start of every GEMM workspace (two int32 per CTA,
# at most 1024 CTAs): kCounterBytes in awqb_gemm.cu.
COUNTER_BYTES = 8192

workspace_pool = _WorkspacePool()


_WS_BYTES: Dict[Tuple[int, int, int, int, int, int], int] = {}


def gemm_workspace_bytes(M: int, K: int, N: int, G: int, ntok: int = 0, ctas: int = 0) -> int:
    key = (M, K, N, G, ntok, ctas)
    v = _WS_BYTES.get(key)
    if v is None:
        out = c_i64(0)
        call("awqb_gemm_workspace_bytes_ex", M, K, N, G, ntok, ctas, ctypes.byref(out))
        v = _WS_BYTES[key] = out.value
    return v


def gemm_plan(M: int, K: int, N: int, G: int, ntok: int = 0, ctas: int = 0) -> Dict[str, int]:
    """The launch the GEMM makes for these sizes: token tile, CTAs, cluster size."""
    t, c, s = ctypes.c_int(0), c_i64(0), ctypes.c_int(0)
    call("awqb_gemm_plan", M, K, N, G, ntok, ctas, ctypes.byref(t), ctypes.byref(c), ctypes.byref(s))
    return {"ntok": t.value, "ctas": c.value, "cluster": s.value}


# ---------------------------------------------------------------- GEMM
def gemm(x: torch.Tensor, blob: torch.Tensor, K: int, N: int, G: int,
         bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
         ntok: int = 0, ctas: int = 0, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[..., N] = x[..., K] @ dequant(blob) (+ bias), fp32 accumulation."""
    if x.shape[-1] != K:
        raise ValueError(f"x has {x.shape[-1]} features, expected K={K}")
    x2 = x if x.dim() == 2 else x.reshape(-1, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M = x2.shape[0]
    code = DTYPE_CODE.get(x.dtype)
    if code is None:
        raise ValueError(f"activation dtype {x.dtype} not supported (float16 or bfloat16)")
    if not (x2.is_cuda and blob.is_cuda):
        raise ValueError("tensors must live on a CUDA device (there is no CPU path)")
    di = x2.get_device()
    if blob.get_device() != di or not blob.is_contiguous():
        raise ValueError("blob must be a contiguous tensor on the activations' device")
    if bias is not None:
        if not bias.is_cuda or bias.get_device() != di or bias.dtype != x.dtype or bias.numel() != N \
                or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous [N] tensor in the activation dtype on the same device")
    if out is None:
        out = torch.empty((M, N), dtype=x.dtype, device=x2.device)
    elif (out.shape[-1] != N or out.numel() != M * N or out.dtype != x.dtype or not out.is_contiguous()
          or not out.is_cuda or out.get_device() != di):
        raise ValueError("out must be a contiguous [M, N] tensor of the activation dtype on the same device")
    if M == 0:
        return out.reshape(*x.shape[:-1], N)
    if workspace is None:
        workspace = workspace_pool.get(x2.device, gemm_workspace_bytes(M, K, N, G, ntok, ctas))
    prev = _cur_device()
    if prev != di:
        torch.cuda.set_device(di)
    try:
        check(_gemm_ex()(x2.data_ptr(), M, K, N, G, code, blob.data_ptr(),
                         bias.data_ptr() if bias is not None else None, out.data_ptr(),
                         workspace.data_ptr(), workspace.numel(), ntok, ctas, _raw_stream(di)))
    finally:
        if prev != di:
            torch.cuda.set_device(prev)
    return out if x.dim() == 2 else out.reshape(*x.shape[:-1], N)


def gemv(x: torch.Tensor, blob: torch.Tensor, K: int, N: int, G: int, bias: Optional[torch.Tensor] = None,
         out: Optional[torch.Tensor] = None, features_per_cta: int = 0, warps: int = 0, ring: int = 0,
         silu_mul: bool = False) -> torch.Tensor:
    """The small-batch kernel (1 <= M <= 32) with an explicit feature slice per
    CTA and compute-warp count ((16, 16), (32, 16), (32, 8) or (64, 8); 0 =
    default) and ring depth (1..16; 0 = default). ``gemm`` takes it by itself
    for small M; this entry point exists for tuning and tests. silu_mul:
    interleaved gate/up blob, output [M, N/2]."""
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    dev = _check_cuda(x2, blob)
    n_out = N // 2 if silu_mul else N
    if out is None:
        out = torch.empty((M, n_out), dtype=x.dtype, device=dev)
    with _DeviceGuard(dev):
        call("awqb_gemv_ex", _p(x2), M, K, N, G, _dtype_code(x.dtype), _p(blob), _p(bias), _p(out),
             int(features_per_cta), int(warps), int(ring), int(bool(silu_mul)), _stream(dev))
    return out.reshape(*x.shape[:-1], n_out)


GEMV_MAX_M = 16  # awqb_gemm takes the small-batch kernel up to this many rows


_GEMM_EX = None


def _gemm_ex():
    global _GEMM_EX
    if _GEMM_EX is None:
        _GEMM_EX = lib().awqb_gemm_ex
    return _GEMM_EX


def device_error(clear: bool = True) -> int:
    """Bits set by kernels whose bounded waits gave up (synchronises). With
    clear, a non-zero word is reset by ``clear_device_error``."""
    v = ctypes.c_uint32(0)
    call("awqb_device_error", ctypes.byref(v))
    if clear and v.value:
        clear_device_error()
    return v.value


def clear_device_error() -> None:
    """Reset the device error word and the split-tile counters of every pooled
    workspace: a GEMM that gave up waiting may have left its tile's arrival
    counters non-zero, which later calls sharing the workspace would take for
    other contributors' partials. Synchronises the device."""
    call("awqb_clear_device_error")
    workspace_pool.reset_counters()
    torch.cuda.synchronize()


def abi_version() -> int:
    return lib().awqb_abi_version()


# ---------------------------------------------------------------- MoE
def moe_topk_softmax(logits: torch.Tensor, topk: int, renormalize: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 softmax over router logits [M, E], top-k weights [M, k] and ids [M, k]."""
    lg = logits.float().contiguous()
    dev = _check_cuda(lg)
    M, E = lg.shape
    w = torch.empty((M, topk), dtype=torch.float32, device=dev)
    ids = torch.empty((M, topk), dtype=torch.int32, device=dev)
    with _DeviceGuard(dev):
        call("awqb_moe_topk_softmax", _p(lg), M, E, topk, int(bool(renormalize)), _p(w), _p(ids), _stream(dev))
    return w, ids


def moe_max_padded(numel: int, num_experts: int, block_m: int) -> int:
    return int(lib().awqb_moe_max_padded(numel, num_experts, block_m))


ALIGN_MULTI_CTA_MIN = 8192  # pairs from which the multi-CTA sort is faster (measured on B200)


def moe_align(topk_ids: torch.Tensor, e_begin: int, e_end: int, block_m: int,
              multi_cta: Optional[bool] = None):
    """Expert-sorted (token, k) ids padded per expert to block_m; returns
    (sorted_ids [max_padded], block_expert [max_padded / block_m], num_post_pad [1]).
    multi_cta: None picks by size; True / False force one of the two (identical) sorts."""
    ids = topk_ids.contiguous()
    dev = _check_cuda(ids)
    numel = ids.numel()
    maxp = moe_max_padded(numel, e_end - e_begin, block_m)
    sorted_ids = torch.empty(maxp, dtype=torch.int32, device=dev)
    block_expert = torch.empty((maxp + block_m - 1) // block_m, dtype=torch.int32, device=dev)
    npp = torch.empty(1, dtype=torch.int32, device=dev)
    if multi_cta is None:
        multi_cta = numel >= ALIGN_MULTI_CTA_MIN
    with _DeviceGuard(dev):
        if multi_cta:
            wsb = int(lib().awqb_moe_align_workspace_bytes(numel, e_end - e_begin))
            ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
            call("awqb_moe_align_ex", _p(ids), numel, e_begin, e_end, block_m, _p(sorted_ids), maxp,
                 _p(block_expert), _p(npp), _p(ws), ws.numel(), _stream(dev))
        else:
            call("awqb_moe_align", _p(ids), numel, e_begin, e_end, block_m, _p(sorted_ids), maxp,
                 _p(block_expert), _p(npp), _stream(dev))
    return sorted_ids, block_expert, npp


def moe_gather_rows(x: torch.Tensor, sorted_ids: torch.Tensor, num_post_pad: torch.Tensor, topk: int,
                    numel: int) -> torch.Tensor:
    dev = _check_cuda(x, sorted_ids, num_post_pad)
    rows = sorted_ids.numel()
    K = x.shape[-1]
    out = torch.empty((rows, K), dtype=x.dtype, device=dev)
    with _DeviceGuard(dev):
        call("awqb_moe_gather_rows", _p(x), K, _p(sorted_ids), _p(num_post_pad), numel, topk, rows, _p(out),
             _stream(dev))
    return out


def moe_grouped_gemm(x_sorted: torch.Tensor, blobs: torch.Tensor, K: int, N: int, G: int,
                     block_expert: torch.Tensor, num_post_pad: torch.Tensor, block_m: int,
                     out: torch.Tensor, row_map: Optional[torch.Tensor] = None,
                     row_scale: Optional[torch.Tensor] = None, num_valid: int = 0) -> torch.Tensor:
    """Grouped W4A16 GEMM over expert-sorted rows (blobs: [E, blob_bytes])."""
    dev = _check_cuda(x_sorted, blobs, block_expert, num_post_pad, out)
    rows = x_sorted.shape[0]
    nb = c_i64(0)
    call("awqb_moe_grouped_workspace_bytes", rows, K, N, G, block_m, ctypes.byref(nb))
    ws = workspace_pool.get(dev, nb.value)
    with _DeviceGuard(dev):
        call("awqb_moe_grouped_gemm", _p(x_sorted), rows, K, N, G, _dtype_code(x_sorted.dtype), _p(blobs),
             blobs.stride(0), _p(block_expert), _p(num_post_pad), block_m, _p(row_map), _p(row_scale),
             num_valid, _p(out), out.shape[-1], _p(ws), ws.numel(), _stream(dev))
    return out


_AWQ_SHIFT = (0, 16, 4, 20, 8, 24, 12, 28)  # bit offset of logical column i of a packed word


def _awq_unpack_cols(w: torch.Tensor) -> torch.Tensor:
    """[..., C/8] int32 in AWQ order -> [..., C] uint8 nibbles."""
    sh = torch.tensor(_AWQ_SHIFT, dtype=torch.int32, device=w.device)
    return ((w.unsqueeze(-1) >> sh) & 0xF).to(torch.uint8).reshape(*w.shape[:-1], w.shape[-1] * 8)


def _awq_pack_cols(q: torch.Tensor) -> torch.Tensor:
    """[..., C] nibbles -> [..., C/8] int32 in AWQ order."""
    sh = torch.tensor(_AWQ_SHIFT, dtype=torch.int64, device=q.device)
    w = (q.reshape(*q.shape[:-1], q.shape[-1] // 8, 8).to(torch.int64) << sh).sum(-1)
    return torch.where(w >= 2**31, w - 2**32, w).to(torch.int32)


def interleave_gate_up(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                       bias: Optional[torch.Tensor] = None):
    """Reorder merged gate_up AWQ tensors ([..., K, 2I/8] packed, [..., K/G, 2I]
    scales) so that column 2j is gate column j and column 2j + 1 is up column j
    (the layout of gemm_silu_mul). Nibbles are moved, never changed: the
    dequantised weights are a column permutation of the originals."""
    two_i = scales.shape[-1]
    if two_i % 16 != 0:
        raise ValueError("fused SiLU-and-mul needs the intermediate size to be a multiple of 8")
    I = two_i // 2
    j = torch.arange(I, device=scales.device)
    cols = torch.stack([j, I + j], dim=1).reshape(-1)
    qw = _awq_pack_cols(_awq_unpack_cols(qweight).index_select(-1, cols.to(qweight.device)))
    qz = _awq_pack_cols(_awq_unpack_cols(qzeros).index_select(-1, cols.to(qzeros.device)))
    out = (qw.contiguous(), qz.contiguous(), scales.index_select(-1, cols).contiguous())
    if bias is not None:
        return out + (bias.index_select(-1, cols.to(bias.device)).contiguous(),)
    return out


def gemm_silu_mul(x: torch.Tensor, blob: torch.Tensor, K: int, N: int, G: int,
                  bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """silu(x @ W_gate) * (x @ W_up) -> [..., N/2] from an interleaved gate_up blob."""
    if x.shape[-1] != K:
        raise ValueError(f"x has {x.shape[-1]} features, expected K={K}")
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    code = _dtype_code(x.dtype)
    dev = _check_cuda(x2, blob)
    if out is None:
        out = torch.empty((M, N // 2), dtype=x.dtype, device=dev)
    elif out.numel() != M * (N // 2) or out.dtype != x.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous [M, N/2] tensor of the activation dtype")
    if M == 0:
        return out.reshape(*x.shape[:-1], N // 2)
    if M > SILU_FUSE_MAX_M:
        # Larger token tiles: the epilogue's SiLU work competes with the
        # dequantisers for issue slots (measured slower); run the GEMM and the
        # interleaved SiLU-and-mul kernel instead.
        h = gemm(x2, blob, K, N, G, bias=bias)
        return silu_and_mul(h, out=out.reshape(M, N // 2), interleaved=True).reshape(*x.shape[:-1], N // 2)
    ws = workspace_pool.get(dev, gemm_workspace_bytes(M, K, N, G))
    with _DeviceGuard(dev):
        call("awqb_gemm_silu_mul", _p(x2), M, K, N, G, code, _p(blob), _p(bias), _p(out), _p(ws), ws.numel(),
             _stream(dev))
    return out.reshape(*x.shape[:-1], N // 2)


# Largest batch (rows) for which the gate_up GEMM applies SiLU-and-mul in its
# epilogue (measured on B200: 1.04-1.36x faster up to 32 rows, slower from 64).
SILU_FUSE_MAX_M = 32


def moe_grouped_gemm_silu_mul(x_sorted: torch.Tensor, blobs: torch.Tensor, K: int, N: int, G: int,
                              block_expert: torch.Tensor, num_post_pad: torch.Tensor, block_m: int,
                              out: torch.Tensor) -> torch.Tensor:
    """Expert gate_up GEMM fused with SiLU-and-mul (interleaved w1): out [rows, N/2]."""
    dev = _check_cuda(x_sorted, blobs, block_expert, num_post_pad, out)
    rows = x_sorted.shape[0]
    nb = c_i64(0)
    call("awqb_moe_grouped_workspace_bytes", rows, K, N, G, block_m, ctypes.byref(nb))
    ws = workspace_pool.get(dev, nb.value)
    with _DeviceGuard(dev):
        call("awqb_moe_grouped_gemm_silu_mul", _p(x_sorted), rows, K, N, G, _dtype_code(x_sorted.dtype),
             _p(blobs), blobs.stride(0), _p(block_expert), _p(num_post_pad), block_m, _p(out), out.shape[-1],
             _p(ws), ws.numel(), _stream(dev))
    return out


def silu_and_mul(h: torch.Tensor, rows_dev: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None, interleaved: bool = False) -> torch.Tensor:
    """silu(h[:, :I]) * h[:, I:] in fp32, rounded to h's dtype (interleaved:
    silu(h[:, 0::2]) * h[:, 1::2], the layout of an interleaved gate_up)."""
    dev = _check_cuda(h)
    rows, two_i = h.shape
    I = two_i // 2
    if out is None:
        out = torch.empty((rows, I), dtype=h.dtype, device=dev)
    with _DeviceGuard(dev):
        call("awqb_silu_and_mul_interleaved" if interleaved else "awqb_silu_and_mul", _p(h), rows, _p(rows_dev), I,
             _dtype_code(h.dtype), _p(out), _stream(dev))
    return out


def _check_device(*ts: torch.Tensor) -> torch.device:
    """Same CUDA device for all (layout is checked by the caller)."""
    dev = ts[0].device
    for t in ts:
        if t.device.type != "cuda":
            raise ValueError("tensors must live on a CUDA device (there is no CPU path)")
        if t.device != dev:
            raise ValueError("tensors must live on the same device")
    return dev


def _rows_2d(t: torch.Tensor, N: int) -> Tuple[torch.Tensor, int]:
    """[..., N] -> ([M, N] view of the same memory, row stride in elements)."""
    if t.shape[-1] != N or t.stride(-1) != 1:
        raise ValueError("the last dimension must be the contiguous feature dimension")
    if t.dim() == 2:
        t2 = t
    elif t.is_contiguous():
        t2 = t.view(-1, N)
    else:
        raise ValueError("tensors with more than 2 dimensions must be contiguous")
    return t2, (t2.stride(0) if t2.shape[0] > 1 else N)


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * weight over the last dimension, fp32 inside
    (flashinfer.rmsnorm semantics)."""
    N = x.shape[-1]
    if weight.numel() != N or weight.dtype != x.dtype or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [N] tensor in the activation dtype")
    dev = _check_device(x, weight)
    x2, ldx = _rows_2d(x, N)
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    o2, ldo = _rows_2d(out, N)
    with _DeviceGuard(dev):
        call("awqb_rmsnorm", _p(x2), _p(weight), _p(o2), x2.shape[0], N, ldx, ldo, float(eps),
             _dtype_code(x.dtype), _stream(dev))
    return out


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float) -> None:
    """In place: residual += x; x = rmsnorm(residual) * weight, the norm taken
    over the fp32 sum (flashinfer.fused_add_rmsnorm semantics)."""
    N = x.shape[-1]
    if residual.shape != x.shape or residual.dtype != x.dtype:
        raise ValueError("residual must have the shape and dtype of x")
    if weight.numel() != N or weight.dtype != x.dtype or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [N] tensor in the activation dtype")
    dev = _check_device(x, residual, weight)
    x2, ldx = _rows_2d(x, N)
    r2, ldr = _rows_2d(residual, N)
    with _DeviceGuard(dev):
        call("awqb_fused_add_rmsnorm", _p(x2), _p(r2), _p(weight), x2.shape[0], N, ldx, ldr, float(eps),
             _dtype_code(x.dtype), _stream(dev))


def moe_topk_sum(y3: torch.Tensor, M: int, topk: int, topk_ids: Optional[torch.Tensor], e_begin: int,
                 e_end: int, out: torch.Tensor) -> torch.Tensor:
    dev = _check_cuda(y3, out)
    H = y3.shape[-1]
    with _DeviceGuard(dev):
        call("awqb_moe_topk_sum", _p(y3), M, topk, H, _p(topk_ids), e_begin, e_end, _dtype_code(y3.dtype),
             _p(out), _stream(dev))
    return out
