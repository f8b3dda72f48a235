"""candle_moe: Python mirror of the kozistr/candle-moe Rust API over the candle-moe-b200 C ABI.

The reference crate exposes ``apply_topk_softmax_inplace``, ``Activation``, and
``FusedMoE{num_experts, num_selected_experts, activation}`` with ``FusedMoE::new`` /
``FusedMoE::forward`` (src/lib.rs:124-335).  This module keeps those names, argument meanings
and error cases, with torch CUDA tensors in place of candle tensors, and calls the B200 kernels
through ``libcandle_moe_b200.so`` (include/candle_moe.h).  There is no CPU path: when the shared
library is missing, every call raises.

Extensions beyond the reference API: ``topk_softmax`` (allocating, optional renormalisation),
``route_prep`` (the sort/align step on its own), ``fused_moe`` (status-checked, optional
caller workspace), ``workspace_size``, ``device_error_bits``, ``set_gemm_path`` /
``last_gemm_path``.
"""
from __future__ import annotations

import ctypes
import enum
import os
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcandle_moe_b200.so")
_lib: Optional[ctypes.CDLL] = None

MOE_OK, MOE_ERR_INVALID_ARG, MOE_ERR_UNSUPPORTED, MOE_ERR_CUDA, MOE_ERR_WORKSPACE, \
    MOE_ERR_NO_MEMORY = range(6)


class MoeError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {lib().moe_status_string(status).decode()} (status {status})")


def lib() -> ctypes.CDLL:
    """The loaded C-ABI library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python candle-moe_b200/build.py`; "
                "candle_moe has no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        P, I32, I64, U32, SZ = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32,
                                ctypes.c_size_t)
        L.topk_softmax.argtypes = [P, P, P, P, I32, I32, I32, P]
        L.topk_softmax.restype = None
        L.fused_moe.argtypes = [P, P, P, P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, ctypes.c_int, ctypes.c_int, U32, U32, P]
        L.fused_moe.restype = None
        L.moe_last_status.argtypes = []
        L.moe_last_status.restype = ctypes.c_int
        L.moe_status_string.argtypes = [ctypes.c_int]
        L.moe_status_string.restype = ctypes.c_char_p
        L.moe_topk_softmax_v2.argtypes = [P, P, P, P, I32, I64, I32, I32, P]
        L.moe_topk_softmax_v2.restype = ctypes.c_int
        L.moe_router_project_topk.argtypes = [P, P, I64, I32, I32, I32, I32, U32, P, P, P, P, P]
        L.moe_router_project_topk.restype = ctypes.c_int
        L.moe_route_prep.argtypes = [P, P, I64, I32, I32, P, P, P, P]
        L.moe_route_prep.restype = ctypes.c_int
        L.moe_fused_workspace_size.argtypes = [I64, I32, I32, I32, I32, U32, U32]
        L.moe_fused_workspace_size.restype = SZ
        L.moe_fused_v2.argtypes = [P, P, P, P, P, P, P, I64, I32, I32, I32, I32, I32, U32, U32, P,
                                   SZ, P]
        L.moe_fused_v2.restype = ctypes.c_int
        L.moe_device_error_bits.argtypes = [I32, I32]
        L.moe_device_error_bits.restype = U32
        L.moe_set_gemm_path.argtypes = [I32]
        L.moe_set_gemm_path.restype = I32
        L.moe_last_gemm_path.argtypes = []
        L.moe_last_gemm_path.restype = I32
        L.moe_fused_scatter.argtypes = [P, P, P, P, P, P, P, P, I64, I32, I32, I32, I32, I32, U32,
                                         U32, P]
        L.moe_fused_scatter.restype = ctypes.c_int
        L.moe_ep_dest_groups.argtypes = [P, I64, I32, I32, I32, I64, P, I32, P, P]
        L.moe_ep_dest_groups.restype = ctypes.c_int
        L.moe_ep_pack.argtypes = [P, P, P, I64, P, P, P, I32, I32, I32, I32, U32, P, P, P, P]
        L.moe_ep_pack.restype = ctypes.c_int
        L.moe_ep_entry_flat.argtypes = [P, P, P, I64, P, I32, I32, I32, P, P]
        L.moe_ep_entry_flat.restype = ctypes.c_int
        L.moe_segment_sum_rows.argtypes = [P, P, I64, I32, U32, P, P]
        L.moe_segment_sum_rows.restype = ctypes.c_int
        L.moe_route_prep_ex.argtypes = [P, P, I64, I32, I32, P, P, P, P, P]
        L.moe_route_prep_ex.restype = ctypes.c_int
        L.moe_gather_rows.argtypes = [P, P, I64, I32, U32, P, P]
        L.moe_gather_rows.restype = ctypes.c_int
        L.moe_combine_rows.argtypes = [P, P, I64, I64, I32, I32, U32, P, P]
        L.moe_combine_rows.restype = ctypes.c_int
        L.moe_set_sm_reserve.argtypes = [I32]
        L.moe_set_sm_reserve.restype = I32
        L.moe_kernel_launches.argtypes = []
        L.moe_kernel_launches.restype = I64
        L.moe_phase_timing.argtypes = [I32]
        L.moe_phase_timing.restype = ctypes.c_int
        L.moe_phase_times.argtypes = [P, P]
        L.moe_phase_times.restype = ctypes.c_int
        U8P = ctypes.POINTER(ctypes.c_uint8)
        L.moe_peer_alloc.argtypes = [SZ, ctypes.POINTER(ctypes.c_void_p), U8P]
        L.moe_peer_alloc.restype = ctypes.c_int
        L.moe_peer_free.argtypes = [P]
        L.moe_peer_free.restype = ctypes.c_int
        L.moe_peer_open.argtypes = [U8P, ctypes.POINTER(ctypes.c_void_p)]
        L.moe_peer_open.restype = ctypes.c_int
        L.moe_peer_close.argtypes = [P]
        L.moe_peer_close.restype = ctypes.c_int
        L.moe_copy_async.argtypes = [P, P, SZ, P]
        L.moe_copy_async.restype = ctypes.c_int
        L.moe_peer_signal.argtypes = [ctypes.POINTER(ctypes.c_void_p), I32, U32, P]
        L.moe_peer_signal.restype = ctypes.c_int
        L.moe_peer_wait.argtypes = [P, I32, U32, I64, P]
        L.moe_peer_wait.restype = ctypes.c_int
        PP = ctypes.POINTER(ctypes.c_void_p)
        L.moe_ep_push_pairs.argtypes = [P, P, P, P, I32, P, P, I32, I32, I32, I32, U32, PP, PP,
                                        P, I32, P]
        L.moe_ep_push_pairs.restype = ctypes.c_int
        L.moe_segment_sum_push.argtypes = [P, P, I64, I32, U32, I32, PP,
                                           ctypes.POINTER(ctypes.c_int64), I32, P]
        L.moe_segment_sum_push.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need_cuda(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a cuda tensor")


def _need_contig(t: torch.Tensor, name: str):
    # The reference takes only the start offset of each tensor and ignores its strides
    # (src/lib.rs:393-410), so a permuted view is silently misread there; here it is an error.
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous (row-major)")


_INDEX_DTYPES = (torch.int32, getattr(torch, "uint32", torch.int32))


# ---------------------------------------------------------------------------------------------
# router: src/lib.rs:10-155
# ---------------------------------------------------------------------------------------------

def apply_topk_softmax_inplace(gating_output: torch.Tensor, topk_weight: torch.Tensor,
                               topk_indices: torch.Tensor,
                               token_expert_indices: torch.Tensor) -> None:
    """Softmax over experts, then top-k, written into the three caller tensors
    (src/lib.rs:124-155 -> kernels/topk_softmax.cu:331-353).

    gating_output [T,E] f32; topk_weight [T,k] f32; topk_indices / token_expert_indices [T,k]
    int32 or uint32.  E must be a power of two <= 256.  The reference dispatches on
    topk_weight's dtype but its kernel always reads f32 (src/lib.rs:130-148 vs
    topk_softmax.cu:344), so only f32 is accepted here."""
    for t, n in ((gating_output, "gating_output"), (topk_weight, "topk_weight"),
                 (topk_indices, "topk_indices"), (token_expert_indices, "token_expert_indices")):
        _need_cuda(t, n)
    if any(t.dim() != 2 for t in (gating_output, topk_weight, topk_indices, token_expert_indices)):
        raise ValueError(
            "apply_topk_softmax_inplace expects input tensors of rank 2 "
            f"(w: {tuple(topk_weight.shape)}, i: {tuple(topk_indices.shape)}, "
            f"ei: {tuple(token_expert_indices.shape)}, g: {tuple(gating_output.shape)})")
    if topk_weight.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise TypeError("apply_topk_softmax_inplace is only supported for f32, f16 and bf16 "
                        f"({topk_weight.dtype})")
    if gating_output.dtype != torch.float32 or topk_weight.dtype != torch.float32:
        raise TypeError("the router reads and writes f32 only (gating_output and topk_weight "
                        "must be float32)")
    if topk_indices.dtype not in _INDEX_DTYPES or token_expert_indices.dtype not in _INDEX_DTYPES:
        raise TypeError("topk_indices and token_expert_indices must be int32 or uint32")
    num_tokens, top_k = topk_weight.shape
    num_experts = gating_output.shape[1]
    if num_experts == 0 or (num_experts & (num_experts - 1)) != 0 or num_experts > 256:
        raise ValueError("num_experts should be power of 2 and smaller than 256 "
                         f"(num_experts: {num_experts})")
    if tuple(topk_indices.shape) != (num_tokens, top_k):
        raise ValueError(f"shape mismatch topk_indices {tuple(topk_indices.shape)}, expected "
                         f"{(num_tokens, top_k)}")
    if tuple(token_expert_indices.shape) != (num_tokens, top_k):
        raise ValueError(f"shape mismatch token_expert_indices "
                         f"{tuple(token_expert_indices.shape)}, expected {(num_tokens, top_k)}")
    if gating_output.shape[0] != num_tokens:
        raise ValueError("gating_output and topk_weight disagree on the number of tokens")
    for t, n in ((gating_output, "gating_output"), (topk_weight, "topk_weight"),
                 (topk_indices, "topk_indices"), (token_expert_indices, "token_expert_indices")):
        _need_contig(t, n)
    if num_tokens == 0:
        return
    with torch.cuda.device(gating_output.device):
        lib().topk_softmax(_ptr(gating_output), _ptr(topk_weight), _ptr(topk_indices),
                           _ptr(token_expert_indices), num_experts, num_tokens, top_k,
                           _stream(gating_output.device))
        st = lib().moe_last_status()
    if st != MOE_OK:
        raise MoeError(st, "topk_softmax")


def topk_softmax(gating_output: torch.Tensor, top_k: int, renormalize: bool = False):
    """Allocating router: returns (weights [T,k] f32, indices [T,k] int32,
    token_expert_indices [T,k] int32).  renormalize divides the k weights by their sum."""
    _need_cuda(gating_output, "gating_output")
    _need_contig(gating_output, "gating_output")
    if gating_output.dtype != torch.float32 or gating_output.dim() != 2:
        raise TypeError("gating_output must be a rank-2 float32 tensor")
    T, E = gating_output.shape
    dev = gating_output.device
    w = torch.empty((T, top_k), dtype=torch.float32, device=dev)
    idx = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    src = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = lib().moe_topk_softmax_v2(_ptr(gating_output), _ptr(w), _ptr(idx), _ptr(src), E, T,
                                       top_k, int(renormalize), _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_topk_softmax_v2")
    return w, idx, src


def router_project_topk(hidden: torch.Tensor, gate_proj: torch.Tensor, top_k: int,
                        renormalize: bool = False, return_logits: bool = False):
    """Router logits = hidden . gate_proj^T fused with topk_softmax (the reference's caller
    computes the logits with a Linear first, README.md:67-73).  hidden [T,H] and gate_proj [E,H]
    f16/bf16.  Returns (weights [T,k] f32, indices [T,k] int32, token_expert_indices [T,k]
    int32), plus the f32 logits [T,E] with return_logits."""
    for t, n in ((hidden, "hidden"), (gate_proj, "gate_proj")):
        _need_cuda(t, n)
        _need_contig(t, n)
    if hidden.dim() != 2 or gate_proj.dim() != 2 or gate_proj.shape[1] != hidden.shape[1]:
        raise ValueError("hidden must be [T, H] and gate_proj [E, H]")
    if gate_proj.dtype != hidden.dtype:
        raise TypeError("gate_proj must have hidden's dtype")
    T, H = hidden.shape
    E = gate_proj.shape[0]
    dev = hidden.device
    w = torch.empty((T, top_k), dtype=torch.float32, device=dev)
    idx = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    src = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    logits = torch.empty((T, E), dtype=torch.float32, device=dev) if return_logits else None
    with torch.cuda.device(dev):
        st = lib().moe_router_project_topk(_ptr(hidden), _ptr(gate_proj), T, H, E, top_k,
                                           int(renormalize), fused_moe_internal_dtype(hidden.dtype),
                                           _ptr(w), _ptr(idx), _ptr(src), _ptr(logits),
                                           _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_router_project_topk")
    return (w, idx, src, logits) if return_logits else (w, idx, src)


# ---------------------------------------------------------------------------------------------
# sort / align: kernels/preprocessing.cuh:253-313
# ---------------------------------------------------------------------------------------------

def route_prep(expert_indices: torch.Tensor, routing_weights: torch.Tensor, num_experts: int):
    """Returns (expert_offsets [E+2] int32, sorted_token_ids [T*k] int32, sorted_weights [T*k]
    f32).  Entries past expert_offsets[E] are left unwritten."""
    _need_cuda(expert_indices, "expert_indices")
    _need_contig(expert_indices, "expert_indices")
    _need_contig(routing_weights, "routing_weights")
    T, k = expert_indices.shape
    dev = expert_indices.device
    offsets = torch.empty((num_experts + 2,), dtype=torch.int32, device=dev)
    st_ids = torch.empty((max(T * k, 1),), dtype=torch.int32, device=dev)
    st_w = torch.empty((max(T * k, 1),), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        st = lib().moe_route_prep(_ptr(expert_indices), _ptr(routing_weights), T, k, num_experts,
                                  _ptr(offsets), _ptr(st_ids), _ptr(st_w), _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_route_prep")
    return offsets, st_ids[:T * k], st_w[:T * k]


def route_prep_ex(expert_indices: torch.Tensor, routing_weights: torch.Tensor, num_experts: int):
    """route_prep that also returns sorted_flat (t*k + j of each sorted row): (offsets [E+2],
    sorted_token [T*k], sorted_weight [T*k], sorted_flat [T*k])."""
    _need_cuda(expert_indices, "expert_indices")
    _need_contig(expert_indices, "expert_indices")
    _need_contig(routing_weights, "routing_weights")
    T, k = expert_indices.shape
    dev = expert_indices.device
    n = max(T * k, 1)
    offsets = torch.empty((num_experts + 2,), dtype=torch.int32, device=dev)
    st_ids = torch.empty((n,), dtype=torch.int32, device=dev)
    st_w = torch.empty((n,), dtype=torch.float32, device=dev)
    st_f = torch.empty((n,), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = lib().moe_route_prep_ex(_ptr(expert_indices), _ptr(routing_weights), T, k,
                                     num_experts, _ptr(offsets), _ptr(st_ids), _ptr(st_w),
                                     _ptr(st_f), _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_route_prep_ex")
    return offsets, st_ids[:T * k], st_w[:T * k], st_f[:T * k]


def ep_dest_groups(expert_indices: torch.Tensor, num_experts: int, num_ranks: int,
                   tokens_per_chunk: int, num_chunks: Optional[int] = None):
    """[T, num_ranks] int32 group of each (token, rank) pair (see include/candle_moe.h); with
    num_chunks, also the [num_chunks, num_ranks] int64 (token, slot) assignment counts."""
    _need_contig(expert_indices, "expert_indices")
    T, k = expert_indices.shape
    dev = expert_indices.device
    groups = torch.empty((T, num_ranks), dtype=torch.int32, device=dev)
    asg = None if num_chunks is None else torch.empty((num_chunks, num_ranks), dtype=torch.int64,
                                                      device=dev)
    with torch.cuda.device(dev):
        st = lib().moe_ep_dest_groups(_ptr(expert_indices), T, k, num_experts, num_ranks,
                                      tokens_per_chunk, _ptr(groups), num_chunks or 0, _ptr(asg),
                                      _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_ep_dest_groups")
    return groups if asg is None else (groups, asg)


def ep_pack(x: torch.Tensor, pair_token: torch.Tensor, pair_flat: torch.Tensor,
            expert_indices: torch.Tensor, routing_weights: torch.Tensor, num_experts: int,
            num_ranks: int, num_pairs_device: Optional[torch.Tensor] = None):
    """(rows [U,H], meta [U, 2k] int32, slot_count [U] int32) of the U = pair_token.numel()
    sorted pairs; with num_pairs_device (an int32 on the GPU) only that many are packed and U is
    the capacity."""
    U = pair_token.numel()
    T, k = expert_indices.shape
    H = x.shape[1]
    dev = x.device
    rows = torch.empty((U, H), dtype=x.dtype, device=dev)
    meta = torch.empty((U, 2 * k), dtype=torch.int32, device=dev)
    count = torch.empty((U,), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = lib().moe_ep_pack(_ptr(x), _ptr(pair_token), _ptr(pair_flat), U,
                               _ptr(num_pairs_device), _ptr(expert_indices), _ptr(routing_weights), k, num_experts,
                               num_ranks, H, fused_moe_internal_dtype(x.dtype), _ptr(rows),
                               _ptr(meta), _ptr(count), _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_ep_pack")
    return rows, meta, count


def ep_entry_flat(pair_token, pair_flat, pair_start, expert_indices, num_experts, num_ranks,
                  num_entries):
    """[num_entries] int32: token slot t*k+j of each per-slot contribution, pair by pair."""
    U = pair_token.numel()
    k = expert_indices.shape[1]
    dev = pair_token.device
    flat = torch.empty((num_entries,), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = lib().moe_ep_entry_flat(_ptr(pair_token), _ptr(pair_flat), _ptr(pair_start), U,
                                     _ptr(expert_indices), k, num_experts, num_ranks, _ptr(flat),
                                     _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_ep_entry_flat")
    return flat


def segment_sum_rows(rows_in: torch.Tensor, segment_start: torch.Tensor) -> torch.Tensor:
    """out[r] = sum(rows_in[segment_start[r]:segment_start[r+1]]) (f32 accumulation)."""
    _need_contig(rows_in, "rows_in")
    _need_contig(segment_start, "segment_start")
    R = segment_start.numel() - 1
    H = rows_in.shape[1]
    dev = rows_in.device
    out = torch.empty((R, H), dtype=rows_in.dtype, device=dev)
    with torch.cuda.device(dev):
        st = lib().moe_segment_sum_rows(_ptr(rows_in), _ptr(segment_start), R, H,
                                        fused_moe_internal_dtype(rows_in.dtype), _ptr(out),
                                        _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_segment_sum_rows")
    return out


def gather_rows(src: torch.Tensor, index: torch.Tensor, out: Optional[torch.Tensor] = None):
    """out[r] = src[index[r]] (index int32, on the GPU)."""
    _need_contig(src, "src")
    _need_contig(index, "index")
    rows, H = index.numel(), src.shape[1]
    if out is None:
        out = torch.empty((rows, H), dtype=src.dtype, device=src.device)
    with torch.cuda.device(src.device):
        st = lib().moe_gather_rows(_ptr(src), _ptr(index), rows, H,
                                   fused_moe_internal_dtype(src.dtype), _ptr(out),
                                   _stream(src.device))
    if st != MOE_OK:
        raise MoeError(st, "moe_gather_rows")
    return out


def combine_rows(rows_buf: torch.Tensor, sorted_flat: torch.Tensor, num_tokens: int, top_k: int,
                 out: Optional[torch.Tensor] = None):
    """out[t] = sum over slots j of rows_buf[r] where sorted_flat[r] == t*top_k + j, in slot
    order, f32 accumulation, one rounding."""
    _need_contig(rows_buf, "rows_buf")
    _need_contig(sorted_flat, "sorted_flat")
    rows, H = rows_buf.shape
    dev = rows_buf.device
    if out is None:
        out = torch.empty((num_tokens, H), dtype=rows_buf.dtype, device=dev)
    with torch.cuda.device(dev):
        st = lib().moe_combine_rows(_ptr(rows_buf), _ptr(sorted_flat), rows, num_tokens, top_k, H,
                                    fused_moe_internal_dtype(rows_buf.dtype), _ptr(out),
                                    _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_combine_rows")
    return out


# ---------------------------------------------------------------------------------------------
# fused MoE: src/lib.rs:157-335
# ---------------------------------------------------------------------------------------------

class Activation(enum.IntEnum):
    """src/lib.rs:157-172 (to_int: Silu=0, Gelu=1, Relu=2)."""
    Silu = 0
    Gelu = 1
    Relu = 2

    def to_int(self) -> int:
        return int(self)


def fused_moe_internal_dtype(dtype: torch.dtype) -> int:
    """src/lib.rs:174-182."""
    if dtype == torch.float16:
        return 0
    if dtype == torch.bfloat16:
        return 1
    if dtype == torch.float32:
        return 2
    raise TypeError(f"dtype {dtype} is not supported")


def validate_moe_inputs(input, gate_weights, up_weights, down_weights, routing_weights,
                        expert_indices, num_experts, num_selected_experts, moe_type):
    """src/lib.rs:185-242, same checks and messages; returns (num_tokens, hidden_dim)."""
    if input.dim() != 2:
        raise ValueError(f"input must be rank 2, got {tuple(input.shape)}")
    num_tokens, hidden_dim = input.shape
    if gate_weights.dim() != 3 or up_weights.dim() != 3:
        raise ValueError("gate_weights and up_weights must be rank 3")
    ne_g, hd_g, id_g = gate_weights.shape
    ne_u, hd_u, id_u = up_weights.shape
    if down_weights is not None:
        if down_weights.dim() != 3:
            raise ValueError("down_weights must be rank 3")
        ne_d, id_d, hd_d = down_weights.shape
    else:
        ne_d, id_d, hd_d = num_experts, id_u, hd_u
    if routing_weights.dim() != 2 or expert_indices.dim() != 2:
        raise ValueError("routing_weights and expert_indices must be rank 2")
    nt, nse = routing_weights.shape
    nt2, nse2 = expert_indices.shape
    if ne_g != num_experts or ne_u != num_experts or ne_d != num_experts:
        raise ValueError("Number of experts mismatch")
    if hd_g != hidden_dim or hd_u != hidden_dim:
        raise ValueError("Hidden dimension mismatch for gate/up weights")
    if hd_d != hidden_dim:
        raise ValueError(f"Hidden dimension mismatch for down weights (expected {hidden_dim}, "
                         f"got {hd_d})")
    if id_g != id_u or id_u != id_d:
        raise ValueError(f"Intermediate dimension mismatch (gate: {id_g}, up: {id_u}, "
                         f"down: {id_d})")
    if nt != num_tokens or nt2 != num_tokens:
        raise ValueError("Number of tokens mismatch")
    if nse != num_selected_experts or nse2 != num_selected_experts:
        raise ValueError("Number of selected experts mismatch")
    if moe_type > 1:
        raise ValueError("moe_type must be one of 0 or 1")
    return num_tokens, hidden_dim


def workspace_size(num_tokens: int, hidden_dim: int, intermediate_dim: int, num_experts: int,
                   top_k: int, moe_type: int, dtype: torch.dtype) -> int:
    return int(lib().moe_fused_workspace_size(num_tokens, hidden_dim, intermediate_dim,
                                              num_experts, top_k, moe_type,
                                              fused_moe_internal_dtype(dtype)))


def fused_moe(input, gate_weights, up_weights, down_weights, routing_weights, expert_indices,
              num_experts: int, top_k: int, activation: int, moe_type: int,
              out: Optional[torch.Tensor] = None,
              workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Status-checked fused MoE (moe_fused_v2).  Tensors must already be validated; `out` is
    allocated when not given; `workspace` (uint8, >= workspace_size() bytes) is optional."""
    T, H = input.shape
    I = gate_weights.shape[2]
    dev = input.device
    if out is None:
        out = torch.empty((T, H), dtype=input.dtype, device=dev)
    ws_ptr, ws_bytes = None, 0
    if workspace is not None:
        ws_ptr, ws_bytes = _ptr(workspace), workspace.numel() * workspace.element_size()
    with torch.cuda.device(dev):
        st = lib().moe_fused_v2(_ptr(input), _ptr(gate_weights), _ptr(up_weights),
                                _ptr(down_weights), _ptr(routing_weights), _ptr(expert_indices),
                                _ptr(out), T, H, I, num_experts, top_k, int(activation),
                                moe_type, fused_moe_internal_dtype(input.dtype), ws_ptr, ws_bytes,
                                _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_fused_v2")
    return out


def fused_moe_scatter(input, gate_weights, up_weights, down_weights, routing_weights,
                      expert_indices, out_row, out, num_experts: int, activation: int,
                      moe_type: int) -> torch.Tensor:
    """Weighted contribution of every routed (t, j) written to out[out_row[t*k + j]] (no
    combine).  out must be a [rows, H] tensor of the input's dtype."""
    T, H = input.shape
    I = gate_weights.shape[2]
    k = expert_indices.shape[1]
    dev = input.device
    for n, t in (("input", input), ("gate_weights", gate_weights), ("up_weights", up_weights),
                 ("routing_weights", routing_weights), ("expert_indices", expert_indices),
                 ("out_row", out_row), ("out", out)):
        _need_contig(t, n)
    with torch.cuda.device(dev):
        st = lib().moe_fused_scatter(_ptr(input), _ptr(gate_weights), _ptr(up_weights),
                                     _ptr(down_weights), _ptr(routing_weights),
                                     _ptr(expert_indices), _ptr(out_row), _ptr(out), T, H, I,
                                     num_experts, k, int(activation), moe_type,
                                     fused_moe_internal_dtype(input.dtype), _stream(dev))
    if st != MOE_OK:
        raise MoeError(st, "moe_fused_scatter")
    return out


class FusedMoE:
    """src/lib.rs:244-335."""

    def __init__(self, num_experts: int, num_selected_experts: int,
                 activation: Activation = Activation.Silu):
        self.num_experts = num_experts
        self.num_selected_experts = num_selected_experts
        self.activation = Activation(activation)

    @classmethod
    def new(cls, num_experts: int, num_selected_experts: int, activation: Activation):
        return cls(num_experts, num_selected_experts, activation)

    def forward(self, input: torch.Tensor, gate_weights: torch.Tensor, up_weights: torch.Tensor,
                down_weights: Optional[torch.Tensor], routing_weights: torch.Tensor,
                expert_indices: torch.Tensor, moe_type: int) -> torch.Tensor:
        """input [T,H]; gate/up [E,H,I]; down [E,I,H] (Qwen3, moe_type 0) or None (Nomic,
        moe_type 1); routing_weights [T,k] f32; expert_indices [T,k] int32/uint32.  Returns
        [T,H] in input's dtype."""
        validate_moe_inputs(input, gate_weights, up_weights, down_weights, routing_weights,
                            expert_indices, self.num_experts, self.num_selected_experts, moe_type)
        dt = input.dtype
        fused_moe_internal_dtype(dt)
        tensors = [("input", input), ("gate_weights", gate_weights), ("up_weights", up_weights),
                   ("routing_weights", routing_weights), ("expert_indices", expert_indices)]
        if down_weights is not None:
            tensors.append(("down_weights", down_weights))
        for n, t in tensors:
            _need_cuda(t, n)
            _need_contig(t, n)
        for n, t in (("gate_weights", gate_weights), ("up_weights", up_weights),
                     ("down_weights", down_weights)):
            if t is not None and t.dtype != dt:
                raise TypeError(f"{n} must have the input's dtype {dt}, got {t.dtype}")
        if routing_weights.dtype != torch.float32:
            raise TypeError("routing_weights must be float32")
        if expert_indices.dtype not in _INDEX_DTYPES:
            raise TypeError("expert_indices must be int32 or uint32")
        if moe_type == 0 and down_weights is None:
            raise ValueError("moe_type 0 (Qwen3) needs down_weights")
        return fused_moe(input, gate_weights, up_weights, down_weights, routing_weights,
                         expert_indices, self.num_experts, self.num_selected_experts,
                         self.activation.to_int(), moe_type)


class SparseMoeBlock:
    """The MoE layer a model calls around this library (the router Linear, the softmax top-k and
    the expert FFN of README.md:61-97, as in Qwen3-MoE's and Qwen2-MoE's sparse blocks).

    forward(hidden [T,H]) = the router projection fused with the softmax + top-k
    (router_project_topk, renormalised when norm_topk_prob), then the routed experts
    (FusedMoE.forward), plus -- when shared-expert weights are given -- a shared expert that
    every token goes through (FusedMoE with one expert and k = 1, weighted by
    sigmoid(hidden . shared_expert_gate^T) when that gate is given, else by 1).

    router_weight [E,H]; gate/up [E,H,I]; down [E,I,H] (Qwen3, moe_type 0) or None (Nomic,
    moe_type 1); shared_gate/shared_up [1,H,Is] and shared_down [1,Is,H]; shared_expert_gate
    [1,H].  All in the hidden states' dtype (f16/bf16)."""

    def __init__(self, router_weight, gate_weights, up_weights, down_weights, top_k: int,
                 activation: Activation = Activation.Silu, norm_topk_prob: bool = True,
                 shared_gate=None, shared_up=None, shared_down=None, shared_expert_gate=None):
        self.router_weight = router_weight
        self.gate_weights, self.up_weights, self.down_weights = gate_weights, up_weights, down_weights
        self.moe_type = 0 if down_weights is not None else 1
        self.num_experts = router_weight.shape[0]
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.experts = FusedMoE(self.num_experts, top_k, activation)
        self.shared = None
        if shared_gate is not None:
            if shared_up is None or (self.moe_type == 0 and shared_down is None):
                raise ValueError("a shared expert needs gate, up (and down for moe_type 0)")
            self.shared = (shared_gate, shared_up, shared_down)
            self.shared_moe = FusedMoE(1, 1, activation)
        self.shared_expert_gate = shared_expert_gate

    def forward(self, hidden: torch.Tensor, return_router_logits: bool = False):
        w, idx, _, logits = router_project_topk(hidden, self.router_weight, self.top_k,
                                                renormalize=self.norm_topk_prob,
                                                return_logits=True)
        out = self.experts.forward(hidden, self.gate_weights, self.up_weights, self.down_weights,
                                   w, idx, self.moe_type)
        if self.shared is not None:
            T = hidden.shape[0]
            if self.shared_expert_gate is not None:
                sw = torch.sigmoid(torch.nn.functional.linear(
                    hidden, self.shared_expert_gate).float()).contiguous()
            else:
                sw = torch.ones((T, 1), dtype=torch.float32, device=hidden.device)
            sidx = torch.zeros((T, 1), dtype=torch.int32, device=hidden.device)
            g, u, d = self.shared
            out = out + self.shared_moe.forward(hidden, g, u, d, sw, sidx, self.moe_type)
        return (out, logits) if return_router_logits else out


def device_error_bits(device: int = 0, clear: bool = False) -> int:
    return int(lib().moe_device_error_bits(device, int(clear)))


def set_gemm_path(path: int) -> int:
    """0 automatic (decode kernels for <= 32 tokens, grouped GEMMs above), 1 SIMT only,
    2 tensor cores only, 3 automatic without CTA pairs, 4 automatic with GEMM-1 on CTA pairs too
    and no decode kernels (experimental), 5 automatic without the decode kernels, 6 decode
    kernels at any token count; returns the previous setting."""
    return int(lib().moe_set_gemm_path(path))


def set_sm_reserve(sms: int) -> int:
    """SMs the persistent GEMMs leave free for concurrent kernels; returns the previous value."""
    prev = int(lib().moe_set_sm_reserve(sms))
    if prev < 0:
        raise ValueError(f"sm reserve {sms} out of range")
    return prev


def last_gemm_path() -> int:
    """Kernels of this thread's last fused call: 1 SIMT, 2 grouped GEMMs, 3 decode kernels."""
    return int(lib().moe_last_gemm_path())


def kernel_launches() -> int:
    """Kernels launched by the library so far in this process."""
    return int(lib().moe_kernel_launches())


PHASES = ("route_prep", "gemm1", "gemm2", "combine")


def phase_timing(enable: bool) -> None:
    """Start (resetting the totals) or stop per-phase CUDA-event timing of fused calls."""
    lib().moe_phase_timing(int(enable))


def phase_times():
    """(dict phase -> summed ms, number of timed calls); waits for the recorded events."""
    ms = (ctypes.c_double * 4)()
    calls = ctypes.c_int64(0)
    st = lib().moe_phase_times(ms, ctypes.byref(calls))
    if st != MOE_OK:
        raise MoeError(st, "moe_phase_times")
    return {n: float(ms[i]) for i, n in enumerate(PHASES)}, int(calls.value)


# ---------------------------------------------------------------------------------------------
# peer-mapped buffers and arrival flags (expert-parallel exchange over NVLink)
# ---------------------------------------------------------------------------------------------

PEER_HANDLE_BYTES = 64
ERR_PEER_WAIT = 64  # device error bit set by a peer_wait that ran out of time


def peer_alloc(nbytes: int, device) -> tuple[int, bytes]:
    """Zero-filled device memory on `device` that other processes can map: (pointer, handle)."""
    ptr = ctypes.c_void_p()
    h = (ctypes.c_uint8 * PEER_HANDLE_BYTES)()
    with torch.cuda.device(device):
        st = lib().moe_peer_alloc(nbytes, ctypes.byref(ptr), h)
    if st != MOE_OK:
        raise MoeError(st, f"moe_peer_alloc({nbytes})")
    return int(ptr.value), bytes(h)


def peer_free(ptr: int, device) -> None:
    with torch.cuda.device(device):
        st = lib().moe_peer_free(ctypes.c_void_p(ptr))
    if st != MOE_OK:
        raise MoeError(st, "moe_peer_free")


def peer_open(handle: bytes, device) -> int:
    """Map another process's peer_alloc buffer on `device`; returns the local address."""
    ptr = ctypes.c_void_p()
    h = (ctypes.c_uint8 * PEER_HANDLE_BYTES).from_buffer_copy(handle)
    with torch.cuda.device(device):
        st = lib().moe_peer_open(h, ctypes.byref(ptr))
    if st != MOE_OK:
        raise MoeError(st, "moe_peer_open")
    return int(ptr.value)


def peer_close(ptr: int, device) -> None:
    with torch.cuda.device(device):
        st = lib().moe_peer_close(ctypes.c_void_p(ptr))
    if st != MOE_OK:
        raise MoeError(st, "moe_peer_close")


def copy_async(dst: int, src: int, nbytes: int, stream: torch.cuda.Stream) -> None:
    """Copy nbytes from device address src to dst on `stream` (copy engine; peers allowed)."""
    st = lib().moe_copy_async(ctypes.c_void_p(dst), ctypes.c_void_p(src), nbytes,
                              ctypes.c_void_p(stream.cuda_stream))
    if st != MOE_OK:
        raise MoeError(st, "moe_copy_async")


def peer_signal(flag_addrs, value: int, stream: torch.cuda.Stream) -> None:
    """Release-store `value` into each 32-bit flag at the device addresses flag_addrs."""
    n = len(flag_addrs)
    arr = (ctypes.c_void_p * max(n, 1))(*flag_addrs)
    st = lib().moe_peer_signal(arr, n, value & 0xffffffff, ctypes.c_void_p(stream.cuda_stream))
    if st != MOE_OK:
        raise MoeError(st, "moe_peer_signal")


def peer_wait(flags: int, count: int, value: int, timeout_s: float,
              stream: torch.cuda.Stream) -> None:
    """Stream-ordered wait until the count flags at device address `flags` reach `value`; after
    timeout_s the stream continues and device_error_bits() reports ERR_PEER_WAIT."""
    st = lib().moe_peer_wait(ctypes.c_void_p(flags), count, value & 0xffffffff,
                             int(timeout_s * 1e9), ctypes.c_void_p(stream.cuda_stream))
    if st != MOE_OK:
        raise MoeError(st, "moe_peer_wait")


class _RawDeviceMemory:
    """Exposes nbytes at a device address through __cuda_array_interface__ (no ownership)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 2}


def device_bytes(ptr: int, nbytes: int, device) -> torch.Tensor:
    """A uint8 tensor over memory this module allocated (the caller keeps it alive)."""
    return torch.as_tensor(_RawDeviceMemory(ptr, nbytes), device=device)


def ep_push_pairs(x: torch.Tensor, pair_token: torch.Tensor, pair_flat: torch.Tensor,
                  pair_offsets: torch.Tensor, chunk: int, expert_indices: torch.Tensor,
                  routing_weights: torch.Tensor, num_experts: int, num_ranks: int, dst_rows,
                  dst_meta, slot_count: Optional[torch.Tensor], stream: torch.cuda.Stream,
                  blocks: int = 0) -> None:
    """Dispatch of one chunk fused with the pack (see include/candle_moe.h): rows and metadata go
    straight to the destinations' addresses dst_rows[d] / dst_meta[d] (ints)."""
    T, k = expert_indices.shape
    G = num_ranks
    rows = (ctypes.c_void_p * G)(*dst_rows)
    meta = (ctypes.c_void_p * G)(*dst_meta)
    st = lib().moe_ep_push_pairs(_ptr(x), _ptr(pair_token), _ptr(pair_flat), _ptr(pair_offsets),
                                 chunk, _ptr(expert_indices), _ptr(routing_weights), k,
                                 num_experts, G, x.shape[1], fused_moe_internal_dtype(x.dtype),
                                 rows, meta, _ptr(slot_count), blocks,
                                 ctypes.c_void_p(stream.cuda_stream))
    if st != MOE_OK:
        raise MoeError(st, "moe_ep_push_pairs")


def segment_sum_push(rows_in: torch.Tensor, segment_start: torch.Tensor, dst, first_row,
                     stream: torch.cuda.Stream, blocks: int = 0) -> None:
    """segment_sum_rows whose output rows [first_row[s], first_row[s+1]) go to the address
    dst[s] (ints) instead of a local tensor."""
    G = len(dst)
    R = segment_start.numel() - 1
    d = (ctypes.c_void_p * G)(*dst)
    f = (ctypes.c_int64 * (G + 1))(*first_row)
    st = lib().moe_segment_sum_push(_ptr(rows_in), _ptr(segment_start), R, rows_in.shape[1],
                                    fused_moe_internal_dtype(rows_in.dtype), G, d, f, blocks,
                                    ctypes.c_void_p(stream.cuda_stream))
    if st != MOE_OK:
        raise MoeError(st, "moe_segment_sum_push")
