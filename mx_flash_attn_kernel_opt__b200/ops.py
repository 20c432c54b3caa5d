"""Tensor-level entry points over the C ABI.

`run_kernel` mirrors the reference's Python operator surface
(submission_c500_regions.py:979-995: q, k_cache_paged, v_cache_paged, output,
cache_seqlens, block_table and the nine integer arguments of the C `run_kernel`,
task.md:33-54) with the same argument meaning: the block-table row width is
num_blocks / batch_size, the pool has num_blocks pages and the scale is 1/sqrt(headdim).
It launches on torch's current stream.

`decode` is the general form (explicit scale, any pool size / table stride, several
query tokens, optional append of new tokens); `append_kv` is the append step alone.

Both run only the CUDA library: a missing or non-sm_100 device raises.
"""
import ctypes
import math

import torch

from ._lib import PgqaDecodeArgs, PgqaError, PgqaPlan, check, lib

_workspaces = {}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream_handle(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def workspace_for(batch_size, num_heads, num_heads_k, headdim, page_size, device, seqlen_q=1):
    """A zero-initialised workspace tensor for the decode entry points, cached per device
    (grown when a larger shape needs more)."""
    L = lib()
    dev = torch.device(device)
    with torch.cuda.device(dev):
        need = L.pgqa_workspace_size_v2(batch_size, seqlen_q, num_heads, num_heads_k, headdim,
                                        page_size)
    if need == 0:
        raise PgqaError(L.pgqa_last_status() or 2, "pgqa_workspace_size_v2")
    ws = _workspaces.get(dev.index)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=dev)
        _workspaces[dev.index] = ws
    return ws


FP8 = torch.float8_e4m3fn


def _check_tensors(q, k, v, out, seq_lens, block_table):
    kv_dt = k.dtype if k.dtype in (torch.bfloat16, FP8) else torch.bfloat16
    for name, t, dt in (("q", q, torch.bfloat16), ("k", k, kv_dt),
                        ("v", v, kv_dt), ("out", out, torch.bfloat16),
                        ("seq_lens", seq_lens, torch.int32),
                        ("block_table", block_table, torch.int32)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if t.dtype != dt:
            raise TypeError(f"{name} must be {dt}, got {t.dtype}")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")


def _scale_array(x, Hkv, device):
    """Per-KV-head dequantisation factors as a float32 device tensor (None stays None)."""
    if x is None:
        return None
    if not torch.is_tensor(x):
        x = torch.full((Hkv,), float(x), dtype=torch.float32)
    x = x.to(device=device, dtype=torch.float32).reshape(-1)
    if x.numel() == 1:
        x = x.expand(Hkv)
    if x.numel() != Hkv:
        raise PgqaError(2, "k_scale / v_scale must hold one value or one per KV head")
    return x.contiguous()


def decode(q, k_cache, v_cache, block_table, seq_lens, scale=None, out=None,
           max_seqlen=0, workspace=None, causal=False, k_new=None, v_new=None,
           k_scale=None, v_scale=None, return_lse=False):
    """Paged GQA decode.

    q [B, Hq, D] (one query token) or [B, Sq, Hq, D] bf16; k_cache/v_cache
    [num_pages, P, Hkv, D], bf16 or float8_e4m3fn; block_table [B, stride] int32;
    seq_lens [B] int32.  With Sq > 1 and `causal`, query token i sees keys [0, L - Sq + i].

    k_new / v_new [B, S_new, Hkv, D] (optional, as flash_attn_with_kvcache's k / v, in
    the pools' dtype): the new tokens are first written into the pools at positions
    [L_b, L_b + S_new) and the decode then runs over L_b + S_new keys (seq_lens holds
    the lengths before the append and is not modified).

    FP8 pools: an element of KV head h is worth e4m3 * k_scale[h] (v_scale for V);
    k_scale / v_scale are floats or [Hkv] tensors (None = 1).  Returns out (q's shape),
    or (out, lse) with `return_lse`: lse [B, Hq, Sq] fp32, the natural log of the sum of
    exp(scale * q.k) over the keys each query row sees (-inf for a row that sees none).
    """
    if out is None:
        out = torch.empty_like(q)
    _check_tensors(q, k_cache, v_cache, out, seq_lens, block_table)
    if tuple(out.shape) != tuple(q.shape):
        raise PgqaError(2, f"decode: out {tuple(out.shape)} must have q's shape {tuple(q.shape)}")
    if q.dim() not in (3, 4):
        raise PgqaError(2, "decode: q must be [B, Hq, D] or [B, Sq, Hq, D]")
    devs = {t.device for t in (q, k_cache, v_cache, out, seq_lens, block_table)}
    if len(devs) != 1:
        raise ValueError(f"decode: all tensors must be on one device, got {sorted(map(str, devs))}")
    B = q.shape[0]
    Hq, D = q.shape[-2], q.shape[-1]
    Sq = q.shape[1] if q.dim() == 4 else 1
    num_pages, P, Hkv, Dk = k_cache.shape
    if tuple(v_cache.shape) != tuple(k_cache.shape) or Dk != D:
        raise PgqaError(2, "decode: K/V pool shapes")
    if block_table.dim() != 2 or block_table.shape[0] != B or seq_lens.shape != (B,):
        raise PgqaError(2, "decode: block_table / seq_lens shapes")
    fp8 = k_cache.dtype == FP8
    S_new = _check_new_tokens(k_new, v_new, B, Hkv, D, k_cache.dtype)
    if not fp8 and (k_scale is not None or v_scale is not None):
        raise ValueError("k_scale / v_scale apply to float8_e4m3fn pools only")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if workspace is None:
        workspace = workspace_for(B, Hq, Hkv, D, P, q.device, seqlen_q=Sq)
    L = lib()
    if return_lse:
        lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=q.device)
        ks = _scale_array(k_scale, Hkv, q.device) if fp8 else None
        vs = _scale_array(v_scale, Hkv, q.device) if fp8 else None
        a = PgqaDecodeArgs(
            struct_size=ctypes.sizeof(PgqaDecodeArgs), q=_ptr(q), k_cache=_ptr(k_cache),
            v_cache=_ptr(v_cache), k_new=_ptr(k_new) if S_new else None,
            v_new=_ptr(v_new) if S_new else None, out=_ptr(out), softmax_lse=_ptr(lse),
            seq_lens=_ptr(seq_lens), block_table=_ptr(block_table), batch_size=B,
            seqlen_q=Sq, seqlen_new=S_new, num_heads=Hq, num_heads_k=Hkv, headdim=D,
            page_size=P, num_pages=num_pages, bt_stride=block_table.stride(0),
            max_seqlen=max_seqlen, causal=int(bool(causal)), scale=float(scale),
            kv_format=1 if fp8 else 0, k_scale=_ptr(ks) if ks is not None else None,
            v_scale=_ptr(vs) if vs is not None else None, workspace=_ptr(workspace),
            workspace_bytes=workspace.numel())
        with torch.cuda.device(q.device):
            st = L.pgqa_decode_ex(ctypes.byref(a), _stream_handle(q.device))
        check(st, "pgqa_decode_ex")
        return out, lse
    with torch.cuda.device(q.device):
        if fp8:
            ks = _scale_array(k_scale, Hkv, q.device)
            vs = _scale_array(v_scale, Hkv, q.device)
            st = L.pgqa_decode_fp8(_ptr(q), _ptr(k_cache), _ptr(v_cache),
                                   _ptr(k_new) if S_new else None,
                                   _ptr(v_new) if S_new else None, _ptr(out), _ptr(seq_lens),
                                   _ptr(block_table), B, Sq, S_new, Hq, Hkv, D, P, num_pages,
                                   block_table.stride(0), max_seqlen, int(bool(causal)),
                                   float(scale), _ptr(ks) if ks is not None else None,
                                   _ptr(vs) if vs is not None else None, _ptr(workspace),
                                   workspace.numel(), _stream_handle(q.device))
            what = "pgqa_decode_fp8"
        elif S_new == 0:
            st = L.pgqa_decode_v2(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out),
                                  _ptr(seq_lens), _ptr(block_table), B, Sq, Hq, Hkv, D, P,
                                  num_pages, block_table.stride(0), max_seqlen,
                                  int(bool(causal)), float(scale), _ptr(workspace),
                                  workspace.numel(), _stream_handle(q.device))
            what = "pgqa_decode_v2"
        else:
            st = L.pgqa_decode_kvcache(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(k_new),
                                       _ptr(v_new), _ptr(out), _ptr(seq_lens),
                                       _ptr(block_table), B, Sq, S_new, Hq, Hkv, D, P,
                                       num_pages, block_table.stride(0), max_seqlen,
                                       int(bool(causal)), float(scale), _ptr(workspace),
                                       workspace.numel(), _stream_handle(q.device))
            what = "pgqa_decode_kvcache"
    check(st, what)
    return out


def _check_new_tokens(k_new, v_new, B, Hkv, D, dtype):
    """Validates the appended tokens; returns S_new (0 when none are given)."""
    if k_new is None and v_new is None:
        return 0
    if k_new is None or v_new is None:
        raise ValueError("k_new and v_new go together")
    for name, t in (("k_new", k_new), ("v_new", v_new)):
        if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {dtype} CUDA tensor")
    if k_new.dim() != 4 or tuple(k_new.shape) != tuple(v_new.shape) or \
            k_new.shape[0] != B or k_new.shape[2] != Hkv or k_new.shape[3] != D:
        raise PgqaError(2, "k_new / v_new must be [B, S_new, Hkv, D]")
    return k_new.shape[1]


def append_kv(k_new, v_new, k_cache, v_cache, block_table, seq_lens, workspace=None):
    """Write k_new / v_new [B, S_new, Hkv, D] into the pools (bf16 or float8_e4m3fn) at
    positions [L_b, L_b + S_new) of each sequence (seq_lens = lengths before the append;
    not modified).  Asynchronous on torch's current stream."""
    kv_dt = k_cache.dtype if k_cache.dtype in (torch.bfloat16, FP8) else torch.bfloat16
    for name, t, dt in (("k_cache", k_cache, kv_dt), ("v_cache", v_cache, kv_dt),
                        ("seq_lens", seq_lens, torch.int32),
                        ("block_table", block_table, torch.int32)):
        if not t.is_cuda or t.dtype != dt or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {dt} CUDA tensor")
    num_pages, P, Hkv, D = k_cache.shape
    B = block_table.shape[0]
    S_new = _check_new_tokens(k_new, v_new, B, Hkv, D, k_cache.dtype)
    L = lib()
    fn = L.pgqa_append_kv_fp8 if k_cache.dtype == FP8 else L.pgqa_append_kv
    with torch.cuda.device(k_cache.device):
        st = fn(_ptr(k_new), _ptr(v_new), _ptr(k_cache), _ptr(v_cache), _ptr(seq_lens),
                _ptr(block_table), B, S_new, Hkv, D, P, num_pages, block_table.stride(0),
                _ptr(workspace) if workspace is not None else None,
                _stream_handle(k_cache.device))
    check(st, "pgqa_append_kv")


def run_kernel(q, k_cache_paged, v_cache_paged, output, cache_seqlens, block_table,
               batch_size, seqlen_k, seqlen_q, num_heads, num_heads_k, headdim,
               page_block_size, num_blocks, causal):
    """Reference operator surface (tensors + the C run_kernel integers)."""
    batch_size, num_blocks = int(batch_size), int(num_blocks)
    if batch_size <= 0 or num_blocks % batch_size != 0:
        raise PgqaError(2, "run_kernel: num_blocks must be a multiple of batch_size")
    if int(seqlen_q) < 1 or int(causal) not in (0, 1):
        raise PgqaError(2, "run_kernel: seqlen_q must be >= 1 and causal 0 or 1")
    stride = num_blocks // batch_size
    if int(seqlen_k) > stride * int(page_block_size):
        raise PgqaError(2, "run_kernel: seqlen_k exceeds the block-table capacity")
    shape = (batch_size, int(seqlen_q), int(num_heads), int(headdim))
    q4 = q.view(shape)
    o4 = output.view(shape)
    k = k_cache_paged.view(num_blocks, int(page_block_size), int(num_heads_k), int(headdim))
    v = v_cache_paged.view(num_blocks, int(page_block_size), int(num_heads_k), int(headdim))
    bt = block_table.view(batch_size, stride)
    decode(q4, k, v, bt, cache_seqlens, scale=1.0 / math.sqrt(int(headdim)), out=o4,
           max_seqlen=int(seqlen_k), causal=bool(int(causal)))
    return output


def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, rotary_cos=None,
                            rotary_sin=None, cache_seqlens=None, cache_batch_idx=None,
                            cache_leftpad=None, block_table=None, softmax_scale=None,
                            causal=False, window_size=(-1, -1), softcap=0.0,
                            rotary_interleaved=True, alibi_slopes=None, num_splits=0,
                            return_softmax_lse=False):
    """flash_attn.flash_attn_with_kvcache's argument list (flash-attn 2.8), the operator the
    reference is benchmarked against (task.md:16-26), for the case this library runs: a
    paged cache (`block_table`), per-sequence lengths `cache_seqlens` (int or [B] int32),
    optional new tokens `k` / `v` [B, S_new, Hkv, D] written into the cache in place at
    positions [cache_seqlens[b], cache_seqlens[b] + S_new) first, and the end-aligned
    causal mask.  q is [B, Sq, Hq, D]; returns out of q's shape, or (out, softmax_lse
    [B, Hq, Sq] fp32) with `return_softmax_lse`, as flash-attn does.  `num_splits` is accepted
    and ignored (the split follows the real lengths on the device); `rotary_interleaved`
    only matters with rotary inputs.  Every other option raises NotImplementedError
    instead of being ignored.
    """
    unsupported = []
    if rotary_cos is not None or rotary_sin is not None:
        unsupported.append("rotary embedding (rotary_cos / rotary_sin)")
    if cache_batch_idx is not None:
        unsupported.append("cache_batch_idx")
    if cache_leftpad is not None:
        unsupported.append("cache_leftpad")
    if tuple(window_size) != (-1, -1):
        unsupported.append("window_size (local attention)")
    if softcap:
        unsupported.append("softcap")
    if alibi_slopes is not None:
        unsupported.append("alibi_slopes")
    if block_table is None:
        unsupported.append("a non-paged cache (block_table=None)")
    if unsupported:
        raise NotImplementedError("flash_attn_with_kvcache: not implemented here: "
                                  + ", ".join(unsupported))
    if q.dim() != 4:
        raise ValueError("flash_attn_with_kvcache: q must be [B, Sq, Hq, D]")
    if (k is None) != (v is None):
        raise ValueError("flash_attn_with_kvcache: give both k and v, or neither")
    B = q.shape[0]
    if cache_seqlens is None:
        raise ValueError("flash_attn_with_kvcache: cache_seqlens is required with a paged cache")
    if isinstance(cache_seqlens, int):
        cache_seqlens = torch.full((B,), cache_seqlens, dtype=torch.int32, device=q.device)
    elif cache_seqlens.dtype != torch.int32:
        cache_seqlens = cache_seqlens.to(torch.int32)
    return decode(q, k_cache, v_cache, block_table, cache_seqlens, scale=softmax_scale,
                  causal=bool(causal), k_new=k, v_new=v, return_lse=bool(return_softmax_lse))


def run_kernel_cabi(q, k_cache_paged, v_cache_paged, output, cache_seqlens, block_table,
                    batch_size, seqlen_k, seqlen_q, num_heads, num_heads_k, headdim,
                    page_block_size, num_blocks, causal):
    """Calls the C `run_kernel` symbol exactly as the reference harness does
    (verify_real.py:12-14,32-38: ctypes, 6 pointers + 9 int64, legacy default stream)."""
    L = lib()
    with torch.cuda.device(q.device):
        L.run_kernel(_ptr(q), _ptr(k_cache_paged), _ptr(v_cache_paged), _ptr(output),
                     _ptr(cache_seqlens), _ptr(block_table), int(batch_size), int(seqlen_k),
                     int(seqlen_q), int(num_heads), int(num_heads_k), int(headdim),
                     int(page_block_size), int(num_blocks), int(causal))
        st = L.pgqa_last_status()
    check(st, "run_kernel")
    return output


def check_device_error(workspace=None, device=None):
    """Synchronously read and clear the device error word (raises on error)."""
    L = lib()
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(dev):
        ptr = _ptr(workspace) if workspace is not None else None
        st = L.pgqa_check_device_error(ptr, _stream_handle(dev))
    check(st, "device error word")


def make_plan(batch_size, num_heads, num_heads_k, headdim, page_size, num_sms=0,
              smem_optin=0):
    plan = PgqaPlan()
    st = lib().pgqa_make_plan(batch_size, num_heads, num_heads_k, headdim, page_size,
                              num_sms, smem_optin, ctypes.byref(plan))
    return st, plan
