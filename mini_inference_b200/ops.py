"""Tensor-level wrappers of the C ABI: torch tensors in, kernel launches on the current stream.

Every function here launches sm_100a kernels from ``libpkv.so`` and nothing
else: there is no PyTorch or CPU fallback. Inputs are validated on the host
(shape, dtype, device, last-dim contiguity); index errors found on the device
are written to the caller's status word (see :func:`raise_device_errors`).
"""

from __future__ import annotations

import ctypes
import math

import torch

from ._lib import (PKV_BF16, PKV_DECODE_INPUTS_READY, PKV_DECODE_STATIC_SCRATCH_BYTES, PKV_ERR_WORKSPACE, PKV_F16,
                   PKV_LM_WEIGHT_READY, PkvError, PkvPool, PkvTables, check, lib)

_DTYPES = {torch.float16: PKV_F16, torch.bfloat16: PKV_BF16}


def pkv_dtype(dtype: torch.dtype) -> int:
    if dtype not in _DTYPES:
        raise NotImplementedError(f"the sm_100a kernels take float16 or bfloat16 KV caches, not {dtype}")
    return _DTYPES[dtype]


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("the paged-KV kernels need CUDA tensors (there is no CPU path)")


def _rows_last_contiguous(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def make_pool(k: torch.Tensor, v: torch.Tensor) -> PkvPool:
    """Describe a ``[layers, blocks + 1, kv_heads, block_size, head_dim]`` K/V pair for the C ABI."""
    if k.shape != v.shape or k.dtype != v.dtype or k.dim() != 5:
        raise ValueError("k and v pools must have the same 5-D shape and dtype")
    if not (k.is_contiguous() and v.is_contiguous()):
        raise ValueError("the KV pools must be contiguous")
    layers, nbt, hkv, bs, d = k.shape
    pool = PkvPool(k.data_ptr(), v.data_ptr(), layers, nbt, hkv, bs, d, pkv_dtype(k.dtype))
    pool._keep = (k, v)  # the struct holds raw pointers: keep the tensors alive with it
    return pool


def make_tables(block_tables: torch.Tensor, seq_rows: torch.Tensor | None = None) -> PkvTables:
    """Describe an int32 ``[rows, cols]`` block-table tensor (and optional per-batch row index)."""
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise ValueError("block tables must be a row-major int32 [rows, cols] tensor")
    if seq_rows is not None and (seq_rows.dtype != torch.int32 or not seq_rows.is_contiguous()):
        raise ValueError("seq_rows must be a contiguous int32 tensor")
    rows, cols = block_tables.shape
    tables = PkvTables(block_tables.data_ptr(), block_tables.stride(0), rows, cols, _ptr(seq_rows))
    tables._keep = (block_tables, seq_rows)  # the struct holds raw pointers: keep the tensors alive with it
    return tables


def kv_append(pool: PkvPool, layer: int, k_rows: torch.Tensor, v_rows: torch.Tensor, slot_mapping: torch.Tensor,
              status: torch.Tensor | None = None) -> None:
    """Write rows ``[N, kv_heads, head_dim]`` (any strides; k and v are copied contiguous when
    theirs differ) to ``slot_mapping`` (int64 [N])."""
    _require_cuda(k_rows, v_rows, slot_mapping)
    if k_rows.shape != v_rows.shape:
        raise ValueError("k and v rows must have the same shape")
    if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be a contiguous int64 tensor")
    # One (token, head) stride pair serves both: the reference hands over k as apply_rope's
    # fresh output and v as a view of the projection, whose strides differ.
    if k_rows.stride(-1) != 1 or k_rows.stride() != v_rows.stride():
        k_rows, v_rows = k_rows.contiguous(), v_rows.contiguous()
    n = k_rows.shape[0]
    check(lib.pkv_kv_append(ctypes.byref(pool), layer, k_rows.data_ptr(), v_rows.data_ptr(), n, k_rows.stride(0),
                            k_rows.stride(1), slot_mapping.data_ptr(), _ptr(status), _stream()), "kv_append")


def rope_tables(head_dim: int, max_positions: int, theta: float, dtype: torch.dtype,
                device: torch.device | str) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's cos / sin tables ``[max_positions, head_dim]``, cast to ``dtype``.

    The same torch calls as ``RotaryEmbedding._build`` (engine/model.py:190-199): one
    frequency ``theta^(-2i/d)`` per feature pair computed on the host in float32, positions
    times frequencies on ``device``, the half-table repeated twice, cos and sin in float32,
    then the cast the reference applies per lookup (engine/model.py:208-210). Built on the
    same device, the tables are bit-identical to the reference's.
    """
    exponents = torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim
    inv_freq = (1.0 / (theta**exponents)).to(device)
    positions = torch.arange(max_positions, device=device, dtype=torch.float32)
    freqs = torch.outer(positions, inv_freq)
    angles = torch.cat([freqs, freqs], dim=-1)
    return angles.cos().to(dtype).contiguous(), angles.sin().to(dtype).contiguous()


def rope_append(pool: PkvPool, layer: int, qkv: torch.Tensor, positions: torch.Tensor, cos: torch.Tensor,
                sin: torch.Tensor, num_q_heads: int, q_out: torch.Tensor | None = None, k_out: torch.Tensor | bool = False,
                slot_mapping: torch.Tensor | None = None,
                status: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Rotate q and k of ``qkv`` rows ``[N, (Hq + 2 Hkv) * d]`` by ``positions`` (int64 [N]).

    Returns ``(q_out [N, Hq, d], k_out [N, Hkv, d] or None)``. With ``slot_mapping``
    (int64 [N]) the rotated k and the v columns are also written to the pool at
    ``layer``; ``k_out=True`` allocates the rotated keys, a tensor receives them. The
    results are bit-identical to the reference's ``apply_rope`` on the same tables.
    """
    _require_cuda(qkv, positions, cos, sin, q_out, slot_mapping, k_out if isinstance(k_out, torch.Tensor) else None)
    n = qkv.shape[0]
    hkv, d = pool.num_kv_heads, pool.head_dim
    if qkv.dim() != 2 or qkv.shape[1] != (num_q_heads + 2 * hkv) * d or qkv.stride(1) != 1:
        raise ValueError("qkv must be [N, (Hq + 2 Hkv) * head_dim] with a contiguous last dimension")
    if cos.shape != sin.shape or cos.dim() != 2 or cos.shape[1] != d or not (cos.is_contiguous() and sin.is_contiguous()):
        raise ValueError("cos / sin must be contiguous [max_positions, head_dim] tables")
    if cos.dtype != qkv.dtype or sin.dtype != qkv.dtype or pkv_dtype(qkv.dtype) != pool.dtype:
        raise ValueError("qkv, the tables and the pool must share one dtype")
    if positions.dtype != torch.int64 or not positions.is_contiguous() or positions.numel() != n:
        raise ValueError("positions must be a contiguous int64 tensor with one entry per row")
    if slot_mapping is not None and (slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous()):
        raise ValueError("slot_mapping must be a contiguous int64 tensor")
    if q_out is None:
        q_out = torch.empty(n, num_q_heads, d, dtype=qkv.dtype, device=qkv.device)
    if k_out is True:
        k_out = torch.empty(n, hkv, d, dtype=qkv.dtype, device=qkv.device)
    elif k_out is False:
        k_out = None
    for t in (q_out, k_out):
        if t is not None and t.stride(-1) != 1:
            raise ValueError("q_out / k_out must have a contiguous last dimension")
    check(lib.pkv_rope_append(
        ctypes.byref(pool), layer, qkv.data_ptr(), qkv.stride(0), n, num_q_heads, positions.data_ptr(),
        cos.data_ptr(), sin.data_ptr(), cos.shape[0], q_out.data_ptr(), q_out.stride(0), q_out.stride(1),
        _ptr(k_out), k_out.stride(0) if k_out is not None else 0, k_out.stride(1) if k_out is not None else 0,
        _ptr(slot_mapping), _ptr(status), _stream()), "rope_append")
    return q_out, k_out


def decode_attention_rope(pool: PkvPool, layer: int, tables: PkvTables, qkv: torch.Tensor, cos: torch.Tensor,
                          sin: torch.Tensor, context_lens: torch.Tensor, workspace: torch.Tensor,
                          slot_mapping: torch.Tensor, out: torch.Tensor | None = None, scale: float | None = None,
                          status: torch.Tensor | None = None, inputs_ready: bool = False) -> torch.Tensor:
    """One decode step on one layer from the ``qkv_proj`` rows ``[B, (Hq + 2 Hkv) * d]``, RoPE included.

    q and the new k are rotated in the kernel at position ``context_lens[b] - 1`` on the
    ``cos`` / ``sin`` tables of :func:`rope_tables` (bit-identical to :func:`rope_append`),
    the rotated k and the v columns are appended at ``slot_mapping``, and attention runs:
    one launch for what :func:`rope_append` then :func:`decode_attention` do in two.
    Returns ``out`` ``[B, Hq, d]``.
    """
    _require_cuda(qkv, cos, sin, context_lens, workspace, slot_mapping, out)
    batch = qkv.shape[0]
    hkv, d = pool.num_kv_heads, pool.head_dim
    if qkv.dim() != 2 or qkv.stride(1) != 1 or qkv.shape[1] % d or qkv.shape[1] // d <= 2 * hkv:
        raise ValueError("qkv must be [B, (Hq + 2 Hkv) * head_dim] with a contiguous last dimension")
    hq = qkv.shape[1] // d - 2 * hkv
    if cos.shape != sin.shape or cos.dim() != 2 or cos.shape[1] != d or not (cos.is_contiguous() and sin.is_contiguous()):
        raise ValueError("cos / sin must be contiguous [max_positions, head_dim] tables")
    if cos.dtype != qkv.dtype or sin.dtype != qkv.dtype or pkv_dtype(qkv.dtype) != pool.dtype:
        raise ValueError("qkv, the tables and the pool must share one dtype")
    if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be a contiguous int64 tensor")
    if out is None:
        out = torch.empty(batch, hq, d, dtype=qkv.dtype, device=qkv.device)
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    check(lib.pkv_decode_attention_rope(
        ctypes.byref(pool), layer, ctypes.byref(tables), batch, hq, out.data_ptr(), out.stride(0), out.stride(1),
        qkv.data_ptr(), qkv.stride(0), cos.data_ptr(), sin.data_ptr(), cos.shape[0], slot_mapping.data_ptr(),
        context_lens.data_ptr(), scale, PKV_DECODE_INPUTS_READY if inputs_ready else 0, workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), _ptr(status), _stream()), "decode_attention_rope")
    return out


def decode_workspace_bytes(batch: int, num_kv_heads: int, max_blocks: int, block_size: int, head_dim: int,
                           num_q_heads: int) -> int:
    return int(lib.pkv_decode_workspace_bytes(batch, num_kv_heads, max_blocks, block_size, head_dim, num_q_heads))


def decode_attention(pool: PkvPool, layer: int, tables: PkvTables, q: torch.Tensor, context_lens: torch.Tensor,
                     workspace: torch.Tensor | None, k_new: torch.Tensor | None = None,
                     v_new: torch.Tensor | None = None, slot_mapping: torch.Tensor | None = None,
                     out: torch.Tensor | None = None, scale: float | None = None,
                     status: torch.Tensor | None = None, inputs_ready: bool = False) -> torch.Tensor:
    """One decode step on one layer: q ``[B, Hq, d]`` (any row/head strides), optional fused append.

    Returns ``out`` of shape ``[B, Hq, d]``. ``context_lens`` (int32 [B]) counts the keys
    each row attends to, its new token included. ``inputs_ready`` promises that the
    lengths, tables and cached K/V were complete before the previous kernel in the
    stream began (see PKV_DECODE_INPUTS_READY in include/pkv.h).
    """
    _require_cuda(q, context_lens, k_new, v_new, slot_mapping)
    batch, hq, d = q.shape
    q = _rows_last_contiguous(q)
    if k_new is not None:
        k_new, v_new = _rows_last_contiguous(k_new), _rows_last_contiguous(v_new)
        if k_new.stride() != v_new.stride():
            v_new = v_new.contiguous()
            k_new = k_new.contiguous()
    if out is None:
        out = torch.empty(batch, hq, d, dtype=q.dtype, device=q.device)
    ws_ptr, ws_bytes = (workspace.data_ptr(), workspace.numel() * workspace.element_size()) if workspace is not None \
        else (None, 0)
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    check(lib.pkv_decode_attention(
        ctypes.byref(pool), layer, ctypes.byref(tables), batch, hq, out.data_ptr(), out.stride(0), out.stride(1),
        q.data_ptr(), q.stride(0), q.stride(1), _ptr(k_new), _ptr(v_new),
        k_new.stride(0) if k_new is not None else 0, k_new.stride(1) if k_new is not None else 0,
        _ptr(slot_mapping), context_lens.data_ptr(), scale, PKV_DECODE_INPUTS_READY if inputs_ready else 0,
        ws_ptr, ws_bytes, _ptr(status), _stream()), "decode_attention")
    return out


def decode_reset_workspace(workspace: torch.Tensor) -> None:
    """Zero a decode workspace's ticket counters (after a call that reported an error)."""
    _require_cuda(workspace)
    check(lib.pkv_decode_reset_workspace(workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                                         _stream()), "decode_reset_workspace")


def decode_static_reset() -> None:
    """Zero the current device's static decode scratch tickets (after a static call that reported an error)."""
    check(lib.pkv_decode_static_reset(_stream()), "decode_static_reset")


def decode_static_scratch() -> tuple[int, int]:
    """Device address and size of the current device's static decode scratch."""
    addr, nbytes = ctypes.c_void_p(), ctypes.c_int64()
    check(lib.pkv_decode_static_scratch(ctypes.byref(addr), ctypes.byref(nbytes), _stream()), "decode_static_scratch")
    return int(addr.value or 0), nbytes.value


def decode_attention_static(pool: PkvPool, layer: int, tables: PkvTables, q: torch.Tensor,
                            context_lens: torch.Tensor, out: torch.Tensor, k_new: torch.Tensor | None = None,
                            v_new: torch.Tensor | None = None, slot_mapping: torch.Tensor | None = None,
                            scale: float | None = None, status: torch.Tensor | None = None,
                            inputs_ready: bool = False) -> torch.Tensor:
    """:func:`decode_attention` through the entry point that allocates nothing.

    The library's static per-device scratch replaces the workspace, and this
    wrapper allocates nothing either: ``out`` is required, and tensors whose last
    dimension is strided are refused rather than copied. Calls on one device must
    not overlap on the GPU (they share the scratch). After a call whose status reports an
    error, :func:`decode_static_reset` clears the scratch's tickets.
    """
    _require_cuda(q, context_lens, out, k_new, v_new, slot_mapping)
    batch, hq, d = q.shape
    for t in (q, out, k_new, v_new):
        if t is not None and t.stride(-1) != 1:
            raise ValueError("decode_attention_static copies nothing: the last dimension must be contiguous")
    if k_new is not None and k_new.stride() != v_new.stride():
        raise ValueError("k_new and v_new must have the same strides")
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    status_code = lib.pkv_decode_attention_static(
        ctypes.byref(pool), layer, ctypes.byref(tables), batch, hq, out.data_ptr(), out.stride(0), out.stride(1),
        q.data_ptr(), q.stride(0), q.stride(1), _ptr(k_new), _ptr(v_new),
        k_new.stride(0) if k_new is not None else 0, k_new.stride(1) if k_new is not None else 0,
        _ptr(slot_mapping), context_lens.data_ptr(), scale, PKV_DECODE_INPUTS_READY if inputs_ready else 0,
        _ptr(status), _stream())
    if status_code == PKV_ERR_WORKSPACE:
        raise PkvError(status_code, f"decode_attention_static: this launch needs more than the "
                                    f"{PKV_DECODE_STATIC_SCRATCH_BYTES} bytes of static scratch; "
                                    "use decode_attention with a workspace")
    check(status_code, "decode_attention_static")
    return out


def prefill_attention(pool: PkvPool, layer: int, tables: PkvTables, q: torch.Tensor, cu_seqlens: torch.Tensor,
                      starts: torch.Tensor, max_new_tokens: int, out: torch.Tensor | None = None,
                      scale: float | None = None, status: torch.Tensor | None = None) -> torch.Tensor:
    """Packed prefill on one layer: q ``[N, Hq, d]``; keys come from the pool (append first)."""
    _require_cuda(q, cu_seqlens, starts)
    n, hq, d = q.shape
    q = _rows_last_contiguous(q)
    if out is None:
        out = torch.empty(n, hq, d, dtype=q.dtype, device=q.device)
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    check(lib.pkv_prefill_attention(
        ctypes.byref(pool), layer, ctypes.byref(tables), cu_seqlens.numel() - 1, cu_seqlens.data_ptr(),
        starts.data_ptr(), max_new_tokens, hq, out.data_ptr(), out.stride(0), out.stride(1), q.data_ptr(),
        q.stride(0), q.stride(1), scale, _ptr(status), _stream()), "prefill_attention")
    return out


def lm_head_argmax_workspace(max_batch: int, device: torch.device | str) -> torch.Tensor:
    """A zeroed workspace for :func:`lm_head_argmax` of up to ``max_batch`` rows (each call leaves it zeroed)."""
    nbytes = int(lib.pkv_lm_head_argmax_workspace_bytes(max_batch))
    return torch.zeros((nbytes + 7) // 8, dtype=torch.int64, device=device)


def lm_head_argmax(hidden: torch.Tensor, weight: torch.Tensor, workspace: torch.Tensor,
                   out: torch.Tensor | None = None, max_logits: torch.Tensor | None = None,
                   status: torch.Tensor | None = None, weight_ready: bool = False) -> torch.Tensor:
    """Greedy tokens of ``hidden`` ``[B, H]`` under the LM head ``weight`` ``[V, H]``: int64 ``[B]`` on the device.

    The reference's ``compute_logits(hidden).float().argmax(-1)`` (engine/model.py:321-323,
    engine/sampler.py:27-31) in one kernel: logits rounded to the model dtype, the first index
    among equal maxima, no logits written. ``max_logits`` (float32 ``[B]``, optional) receives
    each row's largest rounded logit. ``weight_ready`` promises that the weight was not written
    by the previous kernel in the stream (see PKV_LM_WEIGHT_READY in include/pkv.h).
    """
    _require_cuda(hidden, weight, workspace, out, max_logits)
    if hidden.dim() != 2 or weight.dim() != 2 or hidden.shape[1] != weight.shape[1]:
        raise ValueError("hidden must be [B, H] and weight [V, H]")
    if hidden.dtype != weight.dtype:
        raise ValueError("hidden and weight must have the same dtype")
    if hidden.stride(1) != 1 or weight.stride(1) != 1:
        raise ValueError("hidden and weight rows must be contiguous")
    batch = hidden.shape[0]
    if out is None:
        out = torch.empty(batch, dtype=torch.int64, device=hidden.device)
    if out.dtype != torch.int64 or out.numel() < batch:
        raise ValueError("out must be int64 with one entry per row")
    if max_logits is not None and (max_logits.dtype != torch.float32 or max_logits.numel() < batch):
        raise ValueError("max_logits must be float32 with one entry per row")
    check(lib.pkv_lm_head_argmax(
        hidden.data_ptr(), hidden.stride(0), batch, weight.data_ptr(), weight.stride(0), weight.shape[0],
        weight.shape[1], pkv_dtype(hidden.dtype), out.data_ptr(), _ptr(max_logits), workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), PKV_LM_WEIGHT_READY if weight_ready else 0, _ptr(status),
        _stream()), "lm_head_argmax")
    return out[:batch]


def _rows2d(t: torch.Tensor, what: str) -> torch.Tensor:
    """``t`` viewed as ``[rows, last]`` without a copy (its rows equally strided, the last dim contiguous)."""
    if t.stride(-1) != 1:
        raise ValueError(f"{what} must have a contiguous last dimension")
    try:
        return t.view(-1, t.shape[-1])
    except RuntimeError as e:
        raise ValueError(f"{what}'s leading dimensions must flatten to one row stride") from e


def add_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """The reference's ``RMSNorm`` (engine/model.py:162-166), after an optional residual add, in one launch.

    With ``residual``: ``residual`` becomes ``residual + x`` (in place, rounded to the dtype, as
    the reference's ``x = x + block(x)``) and the result is the norm of that sum; without it,
    the norm of ``x``. Returns ``out`` (a new tensor shaped like ``x`` unless given).
    """
    _require_cuda(x, weight, residual, out)
    hidden = x.shape[-1]
    if x.dtype == torch.float32:  # split-K partials [splits, rows, hidden] of the block's projection
        return _add_rms_norm_partials(x, weight, eps, residual, out)
    if weight.shape != (hidden,) or weight.dtype != x.dtype or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [hidden] tensor of x's dtype")
    x2 = _rows2d(x, "x")
    r2 = None
    if residual is not None:
        if residual.shape != x.shape or residual.dtype != x.dtype:
            raise ValueError("residual must match x in shape and dtype")
        r2 = _rows2d(residual, "residual")
    if out is None:
        out = torch.empty_like(x)
    if out.shape != x.shape or out.dtype != x.dtype:
        raise ValueError("out must match x in shape and dtype")
    o2 = _rows2d(out, "out")
    check(lib.pkv_add_rms_norm(
        pkv_dtype(x.dtype), x2.data_ptr(), x2.stride(0), _ptr(r2), r2.stride(0) if r2 is not None else 0, _ptr(r2),
        r2.stride(0) if r2 is not None else 0, weight.data_ptr(), o2.data_ptr(), o2.stride(0), x2.shape[0], hidden,
        float(eps), _stream()), "add_rms_norm")
    return out


def _add_rms_norm_partials(parts: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None,
                           out: torch.Tensor | None) -> torch.Tensor:
    """``add_rms_norm`` of ``x = parts.sum(0)`` rounded to the weight's dtype (float32 ``[S, rows, hidden]``)."""
    if parts.dim() != 3 or parts.stride(-1) != 1:
        raise ValueError("partials must be float32 [splits, rows, hidden] with a contiguous last dimension")
    splits, rows, hidden = parts.shape
    if weight.shape != (hidden,) or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [hidden] tensor")
    dt = weight.dtype
    r2 = None
    if residual is not None:
        if residual.shape[-1] != hidden or residual.numel() != rows * hidden or residual.dtype != dt:
            raise ValueError("residual must hold [rows, hidden] of the weight's dtype")
        r2 = _rows2d(residual, "residual")
    if out is None:
        out = torch.empty(rows, hidden, dtype=dt, device=parts.device)
    if out.numel() != rows * hidden or out.dtype != dt:
        raise ValueError("out must hold [rows, hidden] of the weight's dtype")
    o2 = _rows2d(out, "out")
    check(lib.pkv_add_rms_norm_partials(
        pkv_dtype(dt), parts.data_ptr(), parts.stride(1), splits, parts.stride(0), _ptr(r2),
        r2.stride(0) if r2 is not None else 0, _ptr(r2), r2.stride(0) if r2 is not None else 0, weight.data_ptr(),
        o2.data_ptr(), o2.stride(0), rows, hidden, float(eps), _stream()), "add_rms_norm_partials")
    return out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(gate) * up`` of ``gate_up = [..., 2 I]`` (engine/model.py:262-264) in one launch -> ``[..., I]``."""
    _require_cuda(gate_up, out)
    inter = gate_up.shape[-1] // 2
    if gate_up.shape[-1] != 2 * inter:
        raise ValueError("gate_up's last dimension must be even (gate | up)")
    g2 = _rows2d(gate_up, "gate_up")
    if out is None:
        out = torch.empty(*gate_up.shape[:-1], inter, dtype=gate_up.dtype, device=gate_up.device)
    if out.shape != (*gate_up.shape[:-1], inter) or out.dtype != gate_up.dtype:
        raise ValueError("out must be [..., I] of gate_up's dtype")
    o2 = _rows2d(out, "out")
    check(lib.pkv_silu_mul(pkv_dtype(gate_up.dtype), g2.data_ptr(), g2.stride(0), o2.data_ptr(), o2.stride(0),
                           g2.shape[0], inter, _stream()), "silu_mul")
    return out


def build_decode_metadata(tables: PkvTables, lengths: torch.Tensor, block_size: int, scratch_block: int,
                          positions: torch.Tensor, slot_mapping: torch.Tensor, context_lens: torch.Tensor,
                          status: torch.Tensor | None = None) -> None:
    """positions / slot_mapping / context_lens of a decode step from the device table mirror."""
    batch = lengths.numel()
    check(lib.pkv_build_decode_metadata(ctypes.byref(tables), batch, lengths.data_ptr(), block_size, scratch_block,
                                        positions.data_ptr(), slot_mapping.data_ptr(), context_lens.data_ptr(),
                                        _ptr(status), _stream()), "build_decode_metadata")


def build_prefill_metadata(tables: PkvTables, cu_seqlens: torch.Tensor, starts: torch.Tensor, block_size: int,
                           total_tokens: int, positions: torch.Tensor, slot_mapping: torch.Tensor,
                           status: torch.Tensor | None = None) -> None:
    check(lib.pkv_build_prefill_metadata(ctypes.byref(tables), cu_seqlens.numel() - 1, cu_seqlens.data_ptr(),
                                         starts.data_ptr(), block_size, total_tokens, positions.data_ptr(),
                                         slot_mapping.data_ptr(), _ptr(status), _stream()), "build_prefill_metadata")


def update_tables(block_tables: torch.Tensor, updates: torch.Tensor, status: torch.Tensor | None = None) -> None:
    """Apply int32 ``[n, 3]`` (row, column, block) edits to a device table mirror."""
    rows, cols = block_tables.shape
    check(lib.pkv_update_tables(block_tables.data_ptr(), block_tables.stride(0), rows, cols, updates.data_ptr(),
                                updates.shape[0], _ptr(status), _stream()), "update_tables")


def commit_decode(seq_rows: torch.Tensor, lengths: torch.Tensor) -> None:
    check(lib.pkv_commit_decode(seq_rows.data_ptr(), seq_rows.numel(), lengths.data_ptr(), _stream()),
          "commit_decode")


def copy_blocks(pool: PkvPool, src: torch.Tensor, dst: torch.Tensor, status: torch.Tensor | None = None) -> None:
    """Copy whole blocks ``src[i] -> dst[i]`` (int32 device tensors) in every layer, K and V."""
    _require_cuda(src, dst)
    check(lib.pkv_copy_blocks(ctypes.byref(pool), src.data_ptr(), dst.data_ptr(), src.numel(), _ptr(status),
                              _stream()), "copy_blocks")


_STATUS_ERRORS = {
    2: (IndexError, "a block id, slot or position on the device was outside the pool or its table"),
    9: (RuntimeError, "a device-side wait timed out"),
}


def raise_device_errors(status: torch.Tensor) -> None:
    """Read a device status word (synchronises), raise what a kernel recorded, and clear it."""
    code = int(status.item())
    if code:
        status.zero_()
        exc, msg = _STATUS_ERRORS.get(code, (RuntimeError, f"device status {code}"))
        raise exc(msg)
