"""Host side of the B200 KV-cache attention path: ctypes bindings of include/lfm3attn.h and a
per-layer cache object that mirrors how the reference engine owns its KV pools.

The reference engine (Go, internal/model) allocates each layer's paged pool and block table
(engine.go:474-512 allocRuntime), maps logical to physical blocks (engine.go:682-685 SetBlock,
generate.go:281-295 ensureBlock) and passes raw device addresses to its kernels
(prefill.go:464-511, dspark.go:541-621). `LayerCache` does the same with torch-owned device memory;
the library itself never allocates. Every call raises `LFM3AError` on a non-zero return code.

There is no CPU fallback: importing this module loads liblfm3attn.so and fails loudly without it.
"""
from __future__ import annotations

import ctypes
import math
import pathlib
from dataclasses import dataclass

import numpy as np

_HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = _HERE / "liblfm3attn.so"
CUBIN_PATH = _HERE / "cubin" / "lfm3attn_sm100a.cubin"

MODE_F16 = 0
MODE_I8REC = 1
BLOCK_TOKENS = 32
QUANT_BLOCK = 64

OK, EINVAL, ELAUNCH, ETIMEOUT, ECUDA, ENOTSUP, EWORKSPACE, EDEVICE, ENOSPACE = 0, -1, -2, -3, -4, -5, -6, -7, -8


class LFM3AError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"lfm3attn error {code} ({what})")
        self.code = code


class KvLayout(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("block_tokens", ctypes.c_int32),
        ("head_bytes", ctypes.c_int64),
        ("block_bytes", ctypes.c_int64),
    ]


class KvView(ctypes.Structure):
    _fields_ = [
        ("pool", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("pool_blocks", ctypes.c_int64),
        ("layout", KvLayout),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); the exported surface of include/lfm3attn.h.
SIGNATURES = {
    "lfm3a_version": (_I, []),
    "lfm3a_strerror": (ctypes.c_char_p, [_I]),
    "lfm3a_last_error": (ctypes.c_char_p, []),
    "lfm3a_kv_layout_init": (_I, [_I, _I, _I, _I, ctypes.POINTER(KvLayout)]),
    "lfm3a_rope_table": (_I, [ctypes.c_double, ctypes.c_double, _I, _I, _P]),
    "lfm3a_sync": (_I, [_P, _I]),
    "lfm3a_set_wait_limit": (_I, [ctypes.c_uint64]),
    "lfm3a_load_cubin": (_I, [_P, _SZ]),
    "lfm3a_unload_cubin": (_I, []),
    "lfm3a_cubin_launches": (ctypes.c_longlong, []),
    "lfm3a_kv_append": (_I, [ctypes.POINTER(KvView), _P, _P, _I64, _I, _I, _P, _P, _P]),
    "lfm3a_kv_truncate": (_I, [ctypes.POINTER(KvView), _I, _P]),
    "lfm3a_accept": (_I, [_P, _P, _I, _P, _P]),
    "lfm3a_verify_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "lfm3a_verify_splits": (_I, [ctypes.POINTER(KvLayout), _I, _I, _I, _I]),
    "lfm3a_verify_attention": (_I, [ctypes.POINTER(KvView), _P, _I, _I, _I, _I, _P, _P, _P, _SZ, _I, _P]),
    "lfm3a_verify_attention_static": (_I, [ctypes.POINTER(KvView), _P, _I, _I, _I, _I, _P, _P, _I, _P]),
    "lfm3a_verify_partial": (_I, [ctypes.POINTER(KvView), _P, _I, _I, _I, _I, _I, _I, _P, _P, _SZ, _I, _P]),
    "lfm3a_combine": (_I, [_P, _I, _I, _I, _I64, _I64, _P, _P, _P]),
    "lfm3a_verify_round": (_I, [ctypes.POINTER(KvView), _P, _P, _I64, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _SZ, _I,
                                _P]),
    "lfm3a_prefill_i8_splits": (_I, [_I, _I, _I, _I, _I]),
    "lfm3a_prefill_attention_i8": (_I, [ctypes.POINTER(KvView), _P, _I, _I, _I, _I, _I, _P, _P, _SZ, _I, _P]),
    "lfm3a_verify_round_host": (_I, [ctypes.POINTER(KvView), _P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _SZ,
                                     _I, _P, _I]),
    "lfm3a_ring_table": (_I, [_I, _I, _P]),
    "lfm3a_ring_attention": (_I, [ctypes.POINTER(KvView), _P, _I, _I, _I, _I, _P, _P, _SZ, _I, _P]),
    "lfm3a_prefill_workspace_bytes": (_SZ, [_I, _I, _I]),
    "lfm3a_prefill_splits": (_I, [_I, _I, _I, _I, _I]),
    "lfm3a_prefill_attention": (_I, [ctypes.POINTER(KvView), _P, _I, _I, _I, _I, _I, _P, _P, _SZ, _P]),
    "lfm3a_prefill_attention_fused": (_I, [ctypes.POINTER(KvView), _P, _I64, _P, _P, _P, _I64, _I, _I, _I, _I, _I, _P,
                                           _P, _SZ, _P]),
    "lfm3a_quantize_p_u8": (_I, [_P, _I, _P, _P, _P]),
    "lfm3a_quantize_q": (_I, [_P, _I64, _I, _I, _I, _P, _P]),
    "lfm3a_verify_i8_splits": (_I, [ctypes.POINTER(KvLayout), _I, _I, _I, _I]),
    "lfm3a_verify_attention_i8": (_I, [ctypes.POINTER(KvView), _P, _I, _I, _I, _I, _P, _P, _P, _SZ, _I, _P]),
    "lfm3a_g128_packed_bytes": (_I64, [_I, _I]),
    "lfm3a_g128_scale_bytes": (_I64, [_I, _I]),
    "lfm3a_g128_pack": (_I, [_P, _I64, _P, _I64, _I, _I, _P, _P, _P]),
    "lfm3a_g128_quantize": (_I, [_P, _I64, _I, _I, _I, _P, _P, _P]),
    "lfm3a_g128_gemm": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _I64, _P, _I64, _P]),
    "lfm3a_g128_workspace_bytes": (_I64, [_I, _I]),
    "lfm3a_g128_linear": (_I, [_P, _I64, _I, _I, _P, _P, _I, _I, _P, _I64, _P, _I64, _P, _SZ, _P]),
    "lfm3a_gather_region_bytes": (_SZ, [_I, _I, _I]),
    "lfm3a_gather_region_alloc": (_I, [_I, _I, _I, ctypes.POINTER(_P)]),
    "lfm3a_gather_region_free": (_I, [_P]),
    "lfm3a_peer_export": (_I, [_P, _P]),
    "lfm3a_peer_open": (_I, [_P, ctypes.POINTER(_P)]),
    "lfm3a_peer_close": (_I, [_P]),
    "lfm3a_verify_attention_gather": (_I, [ctypes.POINTER(KvView), _P, _I, _I, _I, _I, _P, ctypes.POINTER(_P), _I, _I,
                                           _P, _SZ, _I, _P]),
    "lfm3a_gather_wait": (_I, [_P, _I, _I, _I, _P, _P]),
    "lfm3a_verify_round_gather": (_I, [ctypes.POINTER(KvView), _P, _P, _I64, _P, _P, _P, _I, _I, _I, _I, _P,
                                       ctypes.POINTER(_P), _I, _I, _P, _SZ, _I, _P]),
    "lfm3a_pcache_create": (_I, [_I, _I, _I, ctypes.POINTER(_P)]),
    "lfm3a_pcache_destroy": (None, [_P]),
    "lfm3a_pcache_reset": (None, [_P]),
    "lfm3a_pcache_free_blocks": (_I, [_P]),
    "lfm3a_pcache_cached_blocks": (_I, [_P]),
    "lfm3a_pcache_alloc_slide": (_I, [_P, ctypes.POINTER(_I64)]),
    "lfm3a_pcache_slide_valid": (_I, [_P, _I64]),
    "lfm3a_pcache_alloc_conv": (_I, [_P, ctypes.POINTER(_I64)]),
    "lfm3a_pcache_conv_valid": (_I, [_P, _I64]),
    "lfm3a_pcache_conv_slot": (_I, [_P, _I64]),
    "lfm3a_prefix_salt": (ctypes.c_uint64, [ctypes.c_char_p]),
    "lfm3a_prefix_chain": (ctypes.c_uint64, [ctypes.c_uint64, _P]),
    "lfm3a_pseq_create": (_I, [_P, ctypes.c_char_p, ctypes.POINTER(_P)]),
    "lfm3a_pseq_destroy": (None, [_P, _P]),
    "lfm3a_pseq_reuse": (_I, [_P, _P, _P, _I, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(ctypes.c_int32)]),
    "lfm3a_pseq_ensure": (_I, [_P, _P, _I]),
    "lfm3a_pseq_register": (_I, [_P, _P, _P, _I, _I64]),
    "lfm3a_pseq_release": (_I, [_P, _P]),
    "lfm3a_pseq_blocks": (_I, [_P, _P, _P, _I]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded C-ABI library (loaded on first use; raises when it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise LFM3AError(ECUDA, f"{LIB_PATH} is missing: run __graft_entry__.build()")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def _check(rc: int) -> None:
    if rc != OK:
        detail = lib().lfm3a_last_error().decode(errors="replace")
        raise LFM3AError(rc, f"{lib().lfm3a_strerror(rc).decode()}: {detail}")


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def layout(mode: int, kv_heads: int, head_dim: int, block_tokens: int = BLOCK_TOKENS) -> KvLayout:
    out = KvLayout()
    _check(lib().lfm3a_kv_layout_init(mode, kv_heads, head_dim, block_tokens, ctypes.byref(out)))
    return out


def rope_table(theta: float, factor: float, head_dim: int, positions: int) -> np.ndarray:
    """cos | sin rows per position as fp16 bits (engine.go:428-461 buildRope), computed by the library."""
    out = np.empty((positions, head_dim), dtype=np.uint16)
    _check(lib().lfm3a_rope_table(theta, factor, head_dim, positions, out.ctypes.data))
    return out


def sync(stream=None, timeout_ms: int = 120000) -> None:
    """Bounded wait for the stream plus the device error word (queue.go:292-310 Wait)."""
    _check(lib().lfm3a_sync(_stream(stream), timeout_ms))


_cubin_images = []   # images handed to the driver stay alive while loaded


def load_cubin(path=None) -> None:
    """Loads the committed sm_100a cubin (or `path`) through the CUDA driver API on the current device: from then
    on the library's launches on that device run its kernels (the engine's embedded code objects, kernels/embed.go)."""
    data = pathlib.Path(path or CUBIN_PATH).read_bytes()
    buf = ctypes.create_string_buffer(data, len(data))
    _check(lib().lfm3a_load_cubin(buf, len(data)))
    _cubin_images.append(buf)


def unload_cubin() -> None:
    _check(lib().lfm3a_unload_cubin())


def cubin_launches() -> int:
    """Launches made through the loaded cubin on the current device (-1: none loaded)."""
    return int(lib().lfm3a_cubin_launches())


def set_wait_limit(limit_ns: int = 0) -> None:
    """How long the current device's kernels spin in a bounded wait before raising the device error word
    (0: the default 2 s)."""
    _check(lib().lfm3a_set_wait_limit(limit_ns))


class LayerCache:
    """One layer's paged pool and block table in device memory (engine.go:474-512, 682-685)."""

    def __init__(self, mode: int, kv_heads: int, head_dim: int, capacity_tokens: int, device="cuda",
                 block_table=None, pool_blocks: int | None = None, pool=None):
        """pool: another LayerCache of the same layout whose pool this one shares (a sequence reusing
        another's prefix blocks through its own block table, as the reference's sequences share one
        per-layer pool, engine.go:474-512); else a new zeroed pool of pool_blocks blocks."""
        import torch

        self.layout = layout(mode, kv_heads, head_dim)
        self.mode, self.kv_heads, self.head_dim = mode, kv_heads, head_dim
        self.capacity = capacity_tokens
        logical = (capacity_tokens + BLOCK_TOKENS - 1) // BLOCK_TOKENS
        if pool is not None:
            if pool.layout.block_bytes != self.layout.block_bytes or pool.mode != mode:
                raise LFM3AError(EINVAL, "a shared pool needs the same layout")
            self.pool_blocks, self.pool = pool.pool_blocks, pool.pool
        else:
            self.pool_blocks = pool_blocks if pool_blocks is not None else logical
            self.pool = torch.zeros(self.pool_blocks * self.layout.block_bytes, dtype=torch.uint8, device=device)
        if block_table is None:
            block_table = torch.arange(logical, dtype=torch.int32, device=device)
        self.table = block_table
        self.length = 0
        self.view = KvView(self.pool.data_ptr(), self.table.data_ptr(), self.pool_blocks, self.layout)

    def set_block(self, logical: int, physical: int) -> None:
        self.table[logical] = physical

    def append(self, k, v, pos0: int | None = None, rope=None, k_norm=None, token_stride: int = 0, stream=None) -> None:
        """Stores k, v ([n][kv_heads][head_dim] fp16 device tensors) at positions pos0.. (default: the end)."""
        pos0 = self.length if pos0 is None else pos0
        n = k.shape[0]
        if pos0 + n > self.capacity:
            raise LFM3AError(EINVAL, "append past the cache capacity")
        _check(lib().lfm3a_kv_append(ctypes.byref(self.view), _ptr(k), _ptr(v), token_stride, pos0, n, _ptr(rope),
                                     _ptr(k_norm), _stream(stream)))
        self.length = max(self.length, pos0 + n)

    def truncate(self, new_len: int, stream=None) -> None:
        """Rollback after rejected drafts: the length drops, the tail block's int8 V is re-quantised."""
        _check(lib().lfm3a_kv_truncate(ctypes.byref(self.view), new_len, _stream(stream)))
        self.length = new_len

    def verify(self, q, ctx_len: int, window: int = 0, gate=None, out=None, workspace=None, splits: int = 0,
               stream=None):
        """DSpark verify attention of q ([m][q_heads][head_dim] fp16) over the cache; drafts appended."""
        import torch

        m, qh, d = q.shape
        if out is None:
            out = torch.empty_like(q)
        if splits <= 0:
            splits = verify_splits(self.layout, ctx_len, m, window)
        need = lib().lfm3a_verify_workspace_bytes(m, qh, d, splits)
        if workspace is None and splits > 1:
            workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
        ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
        _check(lib().lfm3a_verify_attention(ctypes.byref(self.view), _ptr(q), m, qh, ctx_len, window, _ptr(gate),
                                            _ptr(out), _ptr(workspace), ws_bytes, splits, _stream(stream)))
        return out

    def verify_round(self, k, v, q, ctx_len: int, rope=None, k_norm=None, window: int = 0, gate=None, out=None,
                     workspace=None, splits: int = 0, stream=None):
        """append(k, v, ctx_len, rope, k_norm) then verify(q, ctx_len, ...) in one library call (the append
        fused into the attention kernel for up to 16 drafts)."""
        import torch

        m, qh, d = q.shape
        if out is None:
            out = torch.empty_like(q)
        if ctx_len + m > self.capacity:
            raise LFM3AError(EINVAL, "append past the cache capacity")
        if splits <= 0:
            splits = verify_splits(self.layout, ctx_len, m, window)
        if workspace is None and splits > 1:
            workspace = torch.zeros(lib().lfm3a_verify_workspace_bytes(m, qh, d, splits), dtype=torch.uint8,
                                    device=q.device)
        ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
        _check(lib().lfm3a_verify_round(ctypes.byref(self.view), _ptr(k), _ptr(v), 0, _ptr(rope), _ptr(k_norm), _ptr(q),
                                        m, qh, ctx_len, window, _ptr(gate), _ptr(out), _ptr(workspace), ws_bytes,
                                        splits, _stream(stream)))
        self.length = max(self.length, ctx_len + m)
        return out

    def verify_round_host(self, host_in, dev_in, host_out, m: int, q_heads: int, ctx_len: int, rope=None,
                          k_norm=None, window: int = 0, gate=None, out=None, workspace=None, splits: int = 0,
                          stream=None, timeout_ms: int = 10000):
        """verify_round with host buffers in one library call: host_in (pinned fp16: the drafts' q, then k, then v,
        contiguous) is copied into dev_in, the round runs, its output is copied into host_out (pinned fp16
        [m][q_heads][head_dim]); the call then waits for the stream up to timeout_ms (> 0), without a limit (0), or
        not at all (< 0)."""
        import torch

        d = self.head_dim
        if out is None:
            out = torch.empty((m, q_heads, d), dtype=torch.float16, device=dev_in.device)
        if ctx_len + m > self.capacity:
            raise LFM3AError(EINVAL, "append past the cache capacity")
        if splits <= 0:
            splits = verify_splits(self.layout, ctx_len, m, window)
        if workspace is None and splits > 1:
            workspace = torch.zeros(lib().lfm3a_verify_workspace_bytes(m, q_heads, d, splits), dtype=torch.uint8,
                                    device=dev_in.device)
        ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
        _check(lib().lfm3a_verify_round_host(ctypes.byref(self.view), _ptr(host_in), _ptr(dev_in), _ptr(rope),
                                             _ptr(k_norm), m, q_heads, ctx_len, window, _ptr(gate), _ptr(out),
                                             _ptr(host_out), _ptr(workspace), ws_bytes, splits, _stream(stream),
                                             timeout_ms))
        self.length = max(self.length, ctx_len + m)
        return out

    def prefill_i8(self, qbuf, tokens: int, q_heads: int, context: int, window: int = 0, out=None, workspace=None,
                   splits: int = 0, stream=None, exact: bool = False):
        """Prefill attention over this MODE_I8REC cache with the reference's arithmetic (prefill_attn.hip:212-505;
        exact: prefill_attn_exact.hip:173-344): qbuf = quantize_q(q) of the tokens (appended at context ..);
        returns fp16 [tokens][q_heads][head_dim]."""
        import torch

        d = self.head_dim
        if out is None:
            out = torch.empty((tokens, q_heads, d), dtype=torch.float16, device=qbuf.device)
        if splits <= 0:
            splits = lib().lfm3a_prefill_i8_splits(tokens, q_heads, context, window, 0)
        if workspace is None:
            workspace = torch.empty(max(1, tokens * q_heads * splits * (d + 2) * 4), dtype=torch.uint8,
                                    device=qbuf.device)
        ws_bytes = workspace.numel() * workspace.element_size()
        _check(lib().lfm3a_prefill_attention_i8(ctypes.byref(self.view), _ptr(qbuf), tokens, q_heads, context, window,
                                                int(exact), _ptr(out), _ptr(workspace), ws_bytes, splits,
                                                _stream(stream)))
        return out

    def verify_i8(self, qbuf, m: int, q_heads: int, ctx_len: int, window: int = 0, gate=None, out=None,
                  workspace=None, splits: int = 0, stream=None):
        """Verify attention over this MODE_I8REC cache with the reference's arithmetic (dspark.hip:1824-2185):
        qbuf = quantize_q(q) of the m tokens; returns fp16 [m][q_heads][head_dim]."""
        import torch

        d = self.head_dim
        if out is None:
            out = torch.empty((m, q_heads, d), dtype=torch.float16, device=qbuf.device)
        if splits <= 0:
            splits = lib().lfm3a_verify_i8_splits(ctypes.byref(self.layout), ctx_len, m, window, 0)
            if splits < 0:
                _check(splits)
        if workspace is None:
            workspace = torch.empty(lib().lfm3a_verify_workspace_bytes(m, q_heads, d, splits), dtype=torch.uint8,
                                    device=qbuf.device)
        ws_bytes = workspace.numel() * workspace.element_size()
        _check(lib().lfm3a_verify_attention_i8(ctypes.byref(self.view), _ptr(qbuf), m, q_heads, ctx_len, window,
                                               _ptr(gate), _ptr(out), _ptr(workspace), ws_bytes, splits,
                                               _stream(stream)))
        return out

    def ring_attention(self, q, ctx_lo: int, ctx_len: int, out=None, workspace=None, splits: int = 0, stream=None):
        """The drafter's ring attention (dspark.hip:1070-1412 with RING): q ([m][q_heads][head_dim] fp16) over
        the live context [ctx_lo, ctx_len) and all m drafts (not causal among them). The cache's block table
        must wrap (ring_table)."""
        import torch

        m, qh, d = q.shape
        if out is None:
            out = torch.empty_like(q)
        if splits <= 0:   # as verify over the live range
            splits = verify_splits(self.layout, ctx_len - ctx_lo, m, 0)
        if workspace is None and splits > 1:
            need = lib().lfm3a_verify_workspace_bytes(m, qh, d, splits)
            workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
        ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
        _check(lib().lfm3a_ring_attention(ctypes.byref(self.view), _ptr(q), m, qh, ctx_lo, ctx_len, _ptr(out),
                                          _ptr(workspace), ws_bytes, splits, _stream(stream)))
        return out

    def verify_partial(self, q, kv_begin: int, kv_end: int, ctx_len: int, window: int = 0, out=None, workspace=None,
                       splits: int = 0, stream=None):
        """This cache shard's log-sum-exp partial [m * q_heads][head_dim + 2] over positions [kv_begin, kv_end)."""
        import torch

        m, qh, d = q.shape
        if out is None:
            out = torch.empty((m * qh, d + 2), dtype=torch.float32, device=q.device)
        if splits <= 0:
            splits = verify_splits(self.layout, kv_end - kv_begin, 1, 0)
        need = lib().lfm3a_verify_workspace_bytes(m, qh, d, splits)
        if workspace is None and splits > 1:
            workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
        ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
        _check(lib().lfm3a_verify_partial(ctypes.byref(self.view), _ptr(q), m, qh, kv_begin, kv_end, ctx_len, window,
                                          _ptr(out), _ptr(workspace), ws_bytes, splits, _stream(stream)))
        return out

    def prefill(self, q, context: int, window: int = 0, exact: bool = False, out=None, workspace=None, stream=None,
                q_norm=None, rope=None, gate=None, q_heads: int | None = None):
        """Causal prefill attention of q at positions context... q: [T][q_heads][head_dim] fp16, or with
        q_heads given any [T][>= q_heads * head_dim] row-strided view of raw projections. q_norm (fp16 [head_dim]),
        rope (a rope_table on the device) and gate (fp16 logits [T][>= q_heads], row-strided) fuse the
        reference's q_norm_rope and gate_mul around the attention."""
        import torch

        d = self.head_dim
        t = q.shape[0]
        qh = q.shape[1] if q_heads is None else q_heads
        q_stride = q.stride(0)
        if out is None:
            out = torch.empty((t, qh, d), dtype=torch.float16, device=q.device)
        need = lib().lfm3a_prefill_workspace_bytes(t, qh, d)
        if workspace is None and need:
            workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
        ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
        gate_stride = gate.stride(0) if gate is not None else 0
        _check(lib().lfm3a_prefill_attention_fused(ctypes.byref(self.view), _ptr(q), q_stride, _ptr(q_norm),
                                                   _ptr(rope), _ptr(gate), gate_stride, t, qh, context, window,
                                                   int(exact), _ptr(out), _ptr(workspace), ws_bytes, _stream(stream)))
        return out

    # -------------------------------------------------------------- host-side inspection
    def logical(self, length: int | None = None) -> dict:
        """Decodes the pool into logical arrays (for checks): see decode_pool."""
        length = self.length if length is None else length
        pool = self.pool.cpu().numpy()
        table = self.table.cpu().numpy()
        return decode_pool(pool, table, self.layout, length)


class PrefixCache:
    """The paged pool's block manager (internal/model/cache.go prefixCache): host memory, in the library.
    full_blocks physical blocks per layer pool, a ring of slide_blocks sliding-window blocks, conv_slots
    conv-state slots (slot 0 running)."""

    def __init__(self, full_blocks: int, slide_blocks: int, conv_slots: int):
        h = _P()
        _check(lib().lfm3a_pcache_create(full_blocks, slide_blocks, conv_slots, ctypes.byref(h)))
        self.handle = h.value

    def close(self) -> None:
        if self.handle:
            lib().lfm3a_pcache_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self) -> None:
        lib().lfm3a_pcache_reset(self.handle)

    @property
    def free_blocks(self) -> int:
        return lib().lfm3a_pcache_free_blocks(self.handle)

    @property
    def cached_blocks(self) -> int:
        return lib().lfm3a_pcache_cached_blocks(self.handle)

    def alloc_slide(self) -> tuple[int, int]:
        ep = _I64()
        slot = lib().lfm3a_pcache_alloc_slide(self.handle, ctypes.byref(ep))
        return slot, ep.value

    def slide_valid(self, epoch: int) -> bool:
        return bool(lib().lfm3a_pcache_slide_valid(self.handle, epoch))

    def alloc_conv(self) -> tuple[int, int]:
        ep = _I64()
        slot = lib().lfm3a_pcache_alloc_conv(self.handle, ctypes.byref(ep))
        return slot, ep.value

    def conv_valid(self, epoch: int) -> bool:
        return bool(lib().lfm3a_pcache_conv_valid(self.handle, epoch))

    def conv_slot(self, epoch: int) -> int:
        rc = lib().lfm3a_pcache_conv_slot(self.handle, epoch)
        if rc < 0:
            _check(rc)
        return rc

    def sequence(self, salt: str = "") -> "PrefixSeq":
        return PrefixSeq(self, salt)


def ring_table(ring_blocks: int, logical_blocks: int) -> np.ndarray:
    """Block table of a ring view: logical block b in ring block b mod ring_blocks (dspark.hip:69-70)."""
    out = np.empty(logical_blocks, dtype=np.int32)
    _check(lib().lfm3a_ring_table(ring_blocks, logical_blocks, out.ctypes.data))
    return out


def prefix_salt(salt: str) -> int:
    """saltSeed (cache.go:138-143)."""
    return lib().lfm3a_prefix_salt(salt.encode())


def prefix_chain(prev: int, tokens) -> int:
    """chainHash (cache.go:145-154) of one 32-token block."""
    t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
    if t.shape != (BLOCK_TOKENS,):
        raise LFM3AError(EINVAL, "a block has 32 tokens")
    return lib().lfm3a_prefix_chain(prev, t.ctypes.data)


class PrefixSeq:
    """One sequence's blocks (generate.go:50-61): reuse, ensure, register, release."""

    def __init__(self, cache: PrefixCache, salt: str = ""):
        h = _P()
        _check(lib().lfm3a_pseq_create(cache.handle, salt.encode(), ctypes.byref(h)))
        self.cache, self.handle = cache, h.value

    def close(self) -> None:
        if self.handle and self.cache.handle:
            lib().lfm3a_pseq_destroy(self.cache.handle, self.handle)
        self.handle = None

    def reuse(self, prompt, window: int = 256, align: int = 1) -> tuple[int, int]:
        """(tokens reused, conv slot to restore). align = 2 for MODE_F16 pools (whole 64-token int8 V blocks)."""
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32))
        n, slot = ctypes.c_int(), ctypes.c_int32()
        _check(lib().lfm3a_pseq_reuse(self.cache.handle, self.handle, p.ctypes.data, p.size, window, align,
                                      ctypes.byref(n), ctypes.byref(slot)))
        return n.value, slot.value

    def ensure(self, logical: int) -> None:
        _check(lib().lfm3a_pseq_ensure(self.cache.handle, self.handle, logical))

    def register(self, tokens, upto: int, conv_epoch: int = -1) -> None:
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        if t.size < upto:
            raise LFM3AError(EINVAL, "register needs upto tokens")
        _check(lib().lfm3a_pseq_register(self.cache.handle, self.handle, t.ctypes.data, upto, conv_epoch))

    def release(self) -> None:
        _check(lib().lfm3a_pseq_release(self.cache.handle, self.handle))

    def blocks(self) -> tuple[np.ndarray, np.ndarray]:
        """(full, slide) logical -> physical block numbers."""
        n = lib().lfm3a_pseq_blocks(self.handle, None, None, 0)
        if n < 0:
            _check(n)
        full = np.zeros(n, dtype=np.int32)
        slide = np.zeros(n, dtype=np.int32)
        lib().lfm3a_pseq_blocks(self.handle, full.ctypes.data, slide.ctypes.data, n)
        return full, slide


def verify_splits(lay: KvLayout, ctx_len: int, m: int, window: int = 0, sm_count: int = 0) -> int:
    rc = lib().lfm3a_verify_splits(ctypes.byref(lay), ctx_len, m, window, sm_count)
    if rc < 0:
        _check(rc)
    return rc


def verify_workspace(m: int, q_heads: int, head_dim: int, splits: int, device="cuda"):
    """A zeroed device workspace of lfm3a_verify_workspace_bytes for a verify call (None for one split)."""
    import torch

    if splits <= 1:
        return None
    return torch.zeros(lib().lfm3a_verify_workspace_bytes(m, q_heads, head_dim, splits), dtype=torch.uint8,
                       device=device)


def combine(partials, rows: int, splits: int, head_dim: int, split_stride: int = 0, row_stride: int = 0, gate=None,
            out=None, stream=None):
    """Log-sum-exp merge of f32 partials (strides in floats; 0 = [rows][splits][head_dim + 2])."""
    import torch

    if out is None:
        out = torch.empty((rows, head_dim), dtype=torch.float16, device=partials.device)
    _check(lib().lfm3a_combine(_ptr(partials), rows, splits, head_dim, split_stride, row_stride, _ptr(gate), _ptr(out),
                               _stream(stream)))
    return out


def accept(best, tokens, state, stream=None) -> None:
    m = tokens.numel()
    _check(lib().lfm3a_accept(_ptr(best), _ptr(tokens), m, _ptr(state), _stream(stream)))


def quantize_q(q, q_heads: int | None = None, head_dim: int | None = None, out=None, stream=None):
    """The reference's query quantiser (prefill_attn.hip:120-135): q fp16 [T][q_heads][head_dim] (or row-strided
    [T][>= q_heads * head_dim] with q_heads, head_dim given) -> qbuf int32 [T * q_heads][head_dim/4 + head_dim/32]."""
    import torch

    t = q.shape[0]
    if q_heads is None:
        q_heads, head_dim = q.shape[1], q.shape[2]
    qbuf = out if out is not None else torch.empty((t * q_heads, head_dim // 4 + head_dim // 32), dtype=torch.int32,
                                                   device=q.device)
    _check(lib().lfm3a_quantize_q(_ptr(q), q.stride(0), t, q_heads, head_dim, _ptr(qbuf), _stream(stream)))
    return qbuf


def quantize_p_u8(p, stream=None):
    import torch

    rows = p.shape[0]
    q = torch.empty((rows, 64), dtype=torch.uint8, device=p.device)
    sc = torch.empty((rows,), dtype=torch.float32, device=p.device)
    _check(lib().lfm3a_quantize_p_u8(_ptr(p), rows, _ptr(q), _ptr(sc), _stream(stream)))
    return q, sc


# ------------------------------------------------------------------ W8A8 linear layers (kernels/gemm.hip)
class G128Operand:
    """An int8 operand of rows x k in g128 tiles with its fp32 group scales, in device memory (torch-owned).
    Weights come from `pack` (row-major int8 + per-row group scales, the layout step of buildPrefillWeights,
    prefill.go:141-215); activations from `quantize` (quantize_pack, gemm.hip:65-103)."""

    def __init__(self, rows: int, k: int, device="cuda"):
        import torch

        self.rows, self.k = rows, k
        nbytes = lib().lfm3a_g128_packed_bytes(rows, k)
        sbytes = lib().lfm3a_g128_scale_bytes(rows, k)
        if nbytes < 0 or sbytes < 0:
            _check(int(nbytes) if nbytes < 0 else int(sbytes))
        self.data = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.scales = torch.empty(sbytes // 4, dtype=torch.float32, device=device)

    @classmethod
    def pack(cls, w, w_scales, stream=None) -> "G128Operand":
        """w: int8 [rows][k] (row stride a multiple of 16 bytes), w_scales: f32 [rows][k / 128], on the device."""
        rows, k = w.shape
        op = cls(rows, k, device=w.device)
        _check(lib().lfm3a_g128_pack(_ptr(w), w.stride(0), _ptr(w_scales), w_scales.stride(0), rows, k, _ptr(op.data),
                                     _ptr(op.scales), _stream(stream)))
        return op

    @classmethod
    def quantize(cls, x, k: int, gated: bool = False, out: "G128Operand | None" = None, stream=None) -> "G128Operand":
        """x: fp16 [rows][>= k] (>= 2k when gated: [gate | up]), row stride a multiple of 8 elements."""
        rows = x.shape[0]
        op = out if out is not None else cls(rows, k, device=x.device)
        _check(lib().lfm3a_g128_quantize(_ptr(x), x.stride(0), rows, k, int(gated), _ptr(op.data), _ptr(op.scales),
                                         _stream(stream)))
        return op


def g128_gemm(a: G128Operand, b: G128Operand, residual=None, out=None, stream=None):
    """out[m][n] = fp16(sum_g sa sb int32-dot [+ residual]) for a (rows x k activations), b (outputs x k weights)."""
    import torch

    if a.k != b.k:
        raise ValueError("operands differ in k")
    if out is None:
        out = torch.empty((a.rows, b.rows), dtype=torch.float16, device=a.data.device)
    _check(lib().lfm3a_g128_gemm(_ptr(a.data), _ptr(a.scales), _ptr(b.data), _ptr(b.scales), a.rows, b.rows, a.k,
                                 _ptr(residual), 0 if residual is None else residual.stride(0), _ptr(out),
                                 out.stride(0), _stream(stream)))
    return out


def g128_workspace_bytes(rows: int, k: int) -> int:
    n = lib().lfm3a_g128_workspace_bytes(rows, k)
    if n < 0:
        _check(int(n))
    return int(n)


def g128_linear(x, w: G128Operand, gated: bool = False, residual=None, out=None, workspace=None, stream=None):
    """One linear layer as the engine's g128 runs it (prefill.go:357-382): quantise x, then the GEMM."""
    import torch

    rows = x.shape[0]
    if out is None:
        out = torch.empty((rows, w.rows), dtype=torch.float16, device=x.device)
    need = g128_workspace_bytes(rows, w.k)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    _check(lib().lfm3a_g128_linear(_ptr(x), x.stride(0), rows, int(gated), _ptr(w.data), _ptr(w.scales), w.rows, w.k,
                                   _ptr(residual), 0 if residual is None else residual.stride(0), _ptr(out),
                                   out.stride(0), _ptr(workspace), workspace.numel() * workspace.element_size(),
                                   _stream(stream)))
    return out


# ------------------------------------------------------------------ page layout (host decoding)
def _f16_section_index(d: int):
    """Index arrays of the MODE_F16 section for s in 0..31, dim in 0..d-1 (see csrc/kv.cuh)."""
    s = np.arange(BLOCK_TOKENS)[:, None]
    dim = np.arange(d)[None, :]
    k_idx = ((s >> 3) * (d // 8) + (dim >> 3)) * 64 + (s & 7) * 8 + (dim & 7)
    v_idx = ((dim >> 3) * 4 + (s >> 3)) * 64 + (dim & 7) * 8 + (s & 7)
    v8_idx = ((dim >> 3) * 2 + (s >> 4)) * 128 + (dim & 7) * 16 + (s & 15)
    return k_idx, v_idx, v8_idx


def decode_pool(pool: np.ndarray, table: np.ndarray, lay: KvLayout, length: int) -> dict:
    """Logical view of `length` tokens of a pool (uint8 bytes).

    MODE_F16 -> K, V [length][kv_heads][head_dim] uint16 (fp16 bits), V8 [64-rounded][kv_heads][head_dim]
    int8 and vscale [blocks of 64][kv_heads] f32. MODE_I8REC -> rec [length][kv_heads][2 * head_dim + 8] uint8.
    """
    h, d = lay.kv_heads, lay.head_dim
    pages = (length + BLOCK_TOKENS - 1) // BLOCK_TOKENS
    if lay.mode == MODE_I8REC:
        rec_bytes = 2 * d + 8
        out = np.zeros((pages * BLOCK_TOKENS, h, rec_bytes), dtype=np.uint8)
        for p in range(pages):
            blk = int(table[p])
            raw = pool[blk * lay.block_bytes:(blk + 1) * lay.block_bytes].reshape(BLOCK_TOKENS, h, rec_bytes)
            out[p * BLOCK_TOKENS:(p + 1) * BLOCK_TOKENS] = raw
        return {"rec": out[:length]}
    k_idx, v_idx, v8_idx = _f16_section_index(d)
    blocks = np.asarray(table[:pages], dtype=np.int64)
    sec = pool[:pool.size // lay.block_bytes * lay.block_bytes].reshape(-1, h, lay.head_bytes)[blocks]   # [pages][h][bytes]
    kk = np.ascontiguousarray(sec[:, :, :64 * d]).view(np.uint16)          # [pages][h][32 d]
    vv = np.ascontiguousarray(sec[:, :, 64 * d:128 * d]).view(np.uint16)
    v8 = np.ascontiguousarray(sec[:, :, 128 * d:160 * d]).view(np.int8)
    K = kk[:, :, k_idx].transpose(0, 2, 1, 3).reshape(pages * BLOCK_TOKENS, h, d)
    V = vv[:, :, v_idx].transpose(0, 2, 1, 3).reshape(pages * BLOCK_TOKENS, h, d)
    V8 = v8[:, :, v8_idx].transpose(0, 2, 1, 3).reshape(pages * BLOCK_TOKENS, h, d)
    page_scale = np.ascontiguousarray(sec[:, :, 160 * d:160 * d + 4]).view(np.float32).reshape(pages, h)
    qblocks = (length + QUANT_BLOCK - 1) // QUANT_BLOCK
    vscale = page_scale[0::2][:qblocks]
    v8_len = min(V8.shape[0], qblocks * QUANT_BLOCK)
    V8_out = np.zeros((qblocks * QUANT_BLOCK, h, d), dtype=np.int8)
    V8_out[:v8_len] = V8[:v8_len]
    return {"K": K[:length], "V": V[:length], "V8": V8_out, "vscale": vscale, "page_scale": page_scale}


@dataclass
class Geometry:
    """Attention geometry: the benchmark's 32/8/64 or the reference model's 16/4/128."""

    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 64

    @property
    def group(self) -> int:
        return self.q_heads // self.kv_heads

    @property
    def qk_scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)


class GatherGroup:
    """This rank's gather region and every rank's region mapped here (the kv-head plan's exchange over
    NVLink peer stores, in place of an all-gather; include/lfm3attn.h, multi-GPU exchange).

    exchange(handle_bytes) -> list of every rank's handle bytes, in rank order (for example through
    torch.distributed.all_gather_object). regions, when given, are existing regions used as the ranks' regions
    directly (all in this process: the one-GPU tests emulate ranks that way)."""

    def __init__(self, world: int, rank: int, rows: int, head_dim: int, exchange=None, regions=None):
        self.world, self.rank, self.rows, self.head_dim = world, rank, rows, head_dim
        self.opened = []
        self.owned = None
        if regions is not None:
            self.region = regions[rank]
            ptrs = list(regions)
        else:
            reg = _P()
            _check(lib().lfm3a_gather_region_alloc(world, rows, head_dim, ctypes.byref(reg)))
            self.region = self.owned = reg.value
            handle = (ctypes.c_char * 64)()
            _check(lib().lfm3a_peer_export(self.region, handle))
            handles = exchange(bytes(handle))
            ptrs = []
            for w in range(world):
                if w == rank:
                    ptrs.append(self.region)
                    continue
                buf = ctypes.create_string_buffer(bytes(handles[w]), 64)
                p = _P()
                _check(lib().lfm3a_peer_open(buf, ctypes.byref(p)))
                self.opened.append(p.value)
                ptrs.append(p.value)
        self.peers = (_P * world)(*ptrs)

    @staticmethod
    def alloc_region(world: int, rows: int, head_dim: int) -> int:
        reg = _P()
        _check(lib().lfm3a_gather_region_alloc(world, rows, head_dim, ctypes.byref(reg)))
        return reg.value

    def verify(self, cache: "LayerCache", q, ctx_len: int, window: int = 0, gate=None, workspace=None, splits: int = 0,
               stream=None) -> None:
        """This rank's verify attention, its output scattered to every rank's region (q: this rank's heads)."""
        import torch

        m, qh, d = q.shape
        if splits <= 0:
            splits = verify_splits(cache.layout, ctx_len, m, window)
        if workspace is None:
            workspace = torch.zeros(lib().lfm3a_verify_workspace_bytes(m, qh, d, splits), dtype=torch.uint8,
                                    device=q.device)
        ws_bytes = workspace.numel() * workspace.element_size()
        _check(lib().lfm3a_verify_attention_gather(ctypes.byref(cache.view), _ptr(q), m, qh, ctx_len, window,
                                                   _ptr(gate), self.peers, self.world, self.rank, _ptr(workspace),
                                                   ws_bytes, splits, _stream(stream)))

    def verify_round(self, cache: "LayerCache", k, v, q, ctx_len: int, rope=None, k_norm=None, window: int = 0,
                     gate=None, workspace=None, splits: int = 0, stream=None) -> None:
        """This rank's verify round (the drafts' append fused into the attention), its output exchanged."""
        import torch

        m, qh, d = q.shape
        if splits <= 0:
            splits = verify_splits(cache.layout, ctx_len, m, window)
        if workspace is None:
            workspace = torch.zeros(lib().lfm3a_verify_workspace_bytes(m, qh, d, splits), dtype=torch.uint8,
                                    device=q.device)
        ws_bytes = workspace.numel() * workspace.element_size()
        _check(lib().lfm3a_verify_round_gather(ctypes.byref(cache.view), _ptr(k), _ptr(v), 0, _ptr(rope), _ptr(k_norm),
                                               _ptr(q), m, qh, ctx_len, window, _ptr(gate), self.peers, self.world,
                                               self.rank, _ptr(workspace), ws_bytes, splits, _stream(stream)))
        cache.length = max(cache.length, ctx_len + m)

    def wait(self, out=None, stream=None) -> None:
        """Waits for every rank's slice of the latest call; writes [world][rows][head_dim] fp16 to out (None: only
        waits)."""
        _check(lib().lfm3a_gather_wait(self.region, self.world, self.rows, self.head_dim, _ptr(out), _stream(stream)))

    def unmap(self) -> None:
        """Unmaps the other ranks' regions (after every rank's last call has finished)."""
        for p in self.opened:
            lib().lfm3a_peer_close(p)
        self.opened = []

    def free(self) -> None:
        """Frees this rank's region: only once every other rank has unmapped it."""
        if self.owned is not None:
            lib().lfm3a_gather_region_free(self.owned)
            self.owned = None

