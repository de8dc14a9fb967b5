"""Tensor-level entry points over the C ABI, for tests, the bench and Python
users that hold their buffers in torch.

These mirror the dispatches the reference's integration models exercise
(integration_tests/models/micro/*/model.py): torch.matmul on f16 operands,
matmul with a transposed RHS, the int8-weight matmul of BASELINE configuration
2 and F.scaled_dot_product_attention. torch provides device memory and the
current stream only; the arithmetic runs in libhxb200.so.
"""
from __future__ import annotations

import torch

from . import _native
from ._native import DTYPE_F16, DTYPE_F32, check


def _stream_ptr(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _rowmajor_ld(t: torch.Tensor, name: str) -> int:
    _require(t.dim() == 2, f"{name} must be 2-D")
    _require(t.stride(1) == 1, f"{name} must have unit inner stride")
    return max(t.stride(0), t.shape[1])


def matmul(a: torch.Tensor, b: torch.Tensor, *, transpose_b: bool = False,
           out_dtype: torch.dtype = torch.float16,
           init: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """C = a @ b (or a @ b.T when transpose_b) (+ init), f16 operands, f32
    accumulation, f16 or f32 result. Semantics of linalg.matmul with a DPS
    init (examples/matmul/matmul.mlir:2-12)."""
    lib = _native.load()
    _require(a.is_cuda and b.is_cuda, "operands must be CUDA tensors")
    _require(a.dtype == torch.float16 and b.dtype == torch.float16, "operands must be f16")
    _require(out_dtype in (torch.float16, torch.float32), "out_dtype must be f16 or f32")
    M, K = a.shape
    if transpose_b:
        N, Kb = b.shape
    else:
        Kb, N = b.shape
    _require(K == Kb, f"contraction mismatch {K} vs {Kb}")
    lda, ldb = _rowmajor_ld(a, "a"), _rowmajor_ld(b, "b")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    ldc = _rowmajor_ld(out, "out")
    if init is not None:
        _require(init.dtype == out.dtype and init.shape == out.shape and
                 init.stride() == out.stride(), "init must match out")
    ws_bytes = lib.hxb_matmul_f16_workspace_bytes(a.data_ptr(), lda, b.data_ptr(), ldb,
                                                  int(transpose_b), M, N, K)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=a.device) if ws_bytes else None
    check(lib.hxb_matmul_f16(
        a.data_ptr(), lda, b.data_ptr(), ldb, int(transpose_b),
        init.data_ptr() if init is not None else None, out.data_ptr(), ldc,
        DTYPE_F16 if out.dtype == torch.float16 else DTYPE_F32, M, N, K,
        ws.data_ptr() if ws is not None else None, ws_bytes, _stream_ptr(a)))
    return out


def w8a16_workspace(device: torch.device | str | None = None) -> torch.Tensor:
    """A zeroed stream-K workspace for matmul_w8a16(..., workspace=) on
    `device` (allocate once, reuse for calls ordered on one stream)."""
    lib = _native.load()
    dev = torch.device(device) if device is not None else torch.device("cuda")
    with torch.cuda.device(dev):
        nbytes = lib.hxb_matmul_w8a16_workspace_bytes(1, 1, 1)
    return torch.zeros(nbytes, dtype=torch.uint8, device=dev)


def matmul_w8a16(a: torch.Tensor, w: torch.Tensor, scale: torch.Tensor,
                 out: torch.Tensor | None = None,
                 residual: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None) -> torch.Tensor:
    """C[M,N] f16 = (a[M,K] f16 @ w[K,N] int8) * scale[N] f16 (+ residual),
    f32 accumulation. With `workspace` (from w8a16_workspace) the dispatch may
    split K across SMs (stream-K) when whole tiles would leave SMs idle."""
    lib = _native.load()
    _require(a.dtype == torch.float16 and w.dtype == torch.int8 and
             scale.dtype == torch.float16, "dtypes must be f16 / int8 / f16")
    M, K = a.shape
    Kw, N = w.shape
    _require(K == Kw and scale.numel() == N and scale.is_contiguous(), "shape mismatch")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=a.device)
    ldc = _rowmajor_ld(out, "out")
    if workspace is not None:
        _require(workspace.is_cuda and workspace.is_contiguous(), "workspace must be a CUDA buffer")
        if residual is not None:
            _require(residual.shape == out.shape and residual.stride() == out.stride() and
                     residual.dtype == torch.float16, "residual must match out")
        check(lib.hxb_matmul_w8a16_streamk(
            a.data_ptr(), _rowmajor_ld(a, "a"), w.data_ptr(), _rowmajor_ld(w, "w"),
            scale.data_ptr(), residual.data_ptr() if residual is not None else None,
            out.data_ptr(), ldc, M, N, K, workspace.data_ptr(),
            workspace.numel() * workspace.element_size(), _stream_ptr(a)))
        return out
    if residual is None:
        check(lib.hxb_matmul_w8a16(a.data_ptr(), _rowmajor_ld(a, "a"), w.data_ptr(),
                                   _rowmajor_ld(w, "w"), scale.data_ptr(), out.data_ptr(),
                                   ldc, M, N, K, _stream_ptr(a)))
    else:
        _require(residual.shape == out.shape and residual.stride() == out.stride() and
                 residual.dtype == torch.float16, "residual must match out")
        check(lib.hxb_matmul_w8a16_residual(a.data_ptr(), _rowmajor_ld(a, "a"), w.data_ptr(),
                                            _rowmajor_ld(w, "w"), scale.data_ptr(),
                                            residual.data_ptr(), out.data_ptr(), ldc, M, N,
                                            K, _stream_ptr(a)))
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
              scale: float | None = None, causal: bool = False,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused scaled-dot-product attention over [..., S, D] f16 tensors."""
    lib = _native.load()
    _require(q.dtype == k.dtype == v.dtype == torch.float16, "q/k/v must be f16")
    _require(q.is_contiguous() and k.is_contiguous() and v.is_contiguous(),
             "q/k/v must be contiguous")
    D = q.shape[-1]
    Sq, Skv = q.shape[-2], k.shape[-2]
    BH = q.numel() // (Sq * D)
    _require(k.numel() // (Skv * D) == BH and v.shape == k.shape, "shape mismatch")
    if scale is None:
        scale = D ** -0.5
    if out is None:
        out = torch.empty_like(q)
    check(lib.hxb_attention_f16(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                BH, Sq, Skv, D, float(scale), int(causal), _stream_ptr(q)))
    return out


def attention_bshd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, batch: int,
                   heads: int, scale: float | None = None, causal: bool = False,
                   out: torch.Tensor | None = None, head_dim: int = 128) -> torch.Tensor:
    """Attention over [batch * S, heads * head_dim] row-major matrices (views
    with unit inner stride, e.g. column blocks of a fused QKV output)."""
    lib = _native.load()
    D = head_dim
    Sq, Skv = q.shape[0] // batch, k.shape[0] // batch
    if scale is None:
        scale = D ** -0.5
    if out is None:
        out = torch.empty((q.shape[0], heads * D), dtype=torch.float16, device=q.device)
    check(lib.hxb_attention_f16_bshd(
        q.data_ptr(), _rowmajor_ld(q, "q"), k.data_ptr(), _rowmajor_ld(k, "k"),
        v.data_ptr(), _rowmajor_ld(v, "v"), out.data_ptr(), _rowmajor_ld(out, "out"),
        batch, heads, Sq, Skv, D, float(scale), int(causal), _stream_ptr(q)))
    return out


ATTN_OUT_LAYOUTS = {"bhsd": 0, "bshd": 1}


def attention_gqa(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *,
                  kv_len: int | None = None, scale: float | None = None, causal: bool = False,
                  q_pos0: int | None = None, out_layout: str = "bhsd",
                  out: torch.Tensor | None = None,
                  workspace: torch.Tensor | None | bool = True) -> torch.Tensor:
    """Grouped-query attention of `query` [B, Hq, q_len, D] over the first
    `kv_len` rows of `k_cache` / `v_cache` [B, Hkv, kv_rows, D]: query head h
    reads KV head h // (Hq // Hkv). The reference's SlicedCacheAttention
    (integration_tests/models/micro/attention-cache-slice-f16/model.py:17-31)
    is attention_gqa(q, k, v, kv_len=context, out_layout="bshd").
    causal masks key j > q_pos0 + i for query i (q_pos0 = the cache position
    of the first query, by default kv_len - q_len).
    out_layout "bhsd" gives [B, Hq, q_len, D], "bshd" [B, q_len, Hq, D].
    workspace: a device tensor for the key split (see
    attention_gqa_workspace_bytes), True to allocate one when the shape
    splits, or None/False to run without the split."""
    lib = _native.load()
    _require(query.dtype == k_cache.dtype == v_cache.dtype == torch.float16,
             "query/k_cache/v_cache must be f16")
    _require(query.dim() == 4 and k_cache.dim() == 4 and v_cache.shape == k_cache.shape,
             "query [B, Hq, q_len, D] and caches [B, Hkv, rows, D] expected")
    _require(query.is_contiguous() and k_cache.is_contiguous() and v_cache.is_contiguous(),
             "query/k_cache/v_cache must be contiguous")
    B, Hq, q_len, D = query.shape
    _require(k_cache.shape[0] == B and k_cache.shape[3] == D, "shape mismatch")
    Hkv, kv_rows = k_cache.shape[1], k_cache.shape[2]
    kv_len = kv_rows if kv_len is None else int(kv_len)
    q_pos0 = kv_len - q_len if q_pos0 is None else int(q_pos0)
    _require(out_layout in ATTN_OUT_LAYOUTS, f"out_layout must be one of {list(ATTN_OUT_LAYOUTS)}")
    if scale is None:
        scale = D ** -0.5
    if out is None:
        shape = (B, Hq, q_len, D) if out_layout == "bhsd" else (B, q_len, Hq, D)
        out = torch.empty(shape, dtype=torch.float16, device=query.device)
    _require(out.is_contiguous() and out.numel() == query.numel(), "out shape mismatch")
    if workspace is True:
        n = attention_gqa_workspace_bytes(B, Hq, Hkv, q_len, kv_len, D)
        workspace = torch.empty(n, dtype=torch.uint8, device=query.device) if n else None
    ws_ptr, ws_bytes = (workspace.data_ptr(), workspace.numel() * workspace.element_size()) \
        if isinstance(workspace, torch.Tensor) else (None, 0)
    check(lib.hxb_attention_gqa_f16(query.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                    out.data_ptr(), B, Hq, Hkv, q_len, q_pos0, kv_len, kv_rows, D,
                                    float(scale), int(causal), ATTN_OUT_LAYOUTS[out_layout],
                                    ws_ptr, ws_bytes, _stream_ptr(query)))
    return out


def attention_gqa_workspace_bytes(batch: int, q_heads: int, kv_heads: int, q_len: int,
                                  kv_len: int, head_dim: int) -> int:
    """Bytes of the key-split workspace attention_gqa uses for this shape on
    the current device (0: it does not split)."""
    return int(_native.load().hxb_attention_gqa_workspace_bytes(batch, q_heads, kv_heads, q_len,
                                                                kv_len, head_dim))


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-5,
            out: torch.Tensor | None = None) -> torch.Tensor:
    lib = _native.load()
    rows, cols = x.shape
    if out is None:
        out = torch.empty_like(x)
    check(lib.hxb_rmsnorm_f16(x.data_ptr(), _rowmajor_ld(x, "x"), gamma.data_ptr(),
                              out.data_ptr(), _rowmajor_ld(out, "out"), rows, cols, float(eps),
                              _stream_ptr(x)))
    return out


def rope_(x: torch.Tensor, heads: int, seq: int, pos0: int = 0,
          theta: float = 10000.0) -> torch.Tensor:
    """In-place RoPE on the first `heads` 128-wide heads of every row."""
    lib = _native.load()
    check(lib.hxb_rope_f16(x.data_ptr(), _rowmajor_ld(x, "x"), x.shape[0], heads, 128, seq,
                           pos0, float(theta), _stream_ptr(x)))
    return x


def swiglu(gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    lib = _native.load()
    rows, two_f = gu.shape
    F = two_f // 2
    if out is None:
        out = torch.empty((rows, F), dtype=torch.float16, device=gu.device)
    check(lib.hxb_swiglu_f16(gu.data_ptr(), _rowmajor_ld(gu, "gu"), out.data_ptr(),
                             _rowmajor_ld(out, "out"), rows, F, _stream_ptr(gu)))
    return out


class DecoderBlockW8:
    """Weights of one int8-weight Llama-style decoder block resident on the
    GPU, and its forward through hxb_decoder_block_w8a16."""

    def __init__(self, *, attn_norm, w_qkv, s_qkv, w_o, s_o, ffn_norm, w_gate_up,
                 s_gate_up, w_down, s_down, heads: int, rms_eps: float = 1e-5,
                 rope_theta: float = 10000.0):
        self.tensors = dict(attn_norm=attn_norm, w_qkv=w_qkv, s_qkv=s_qkv, w_o=w_o, s_o=s_o,
                            ffn_norm=ffn_norm, w_gate_up=w_gate_up, s_gate_up=s_gate_up,
                            w_down=w_down, s_down=s_down)
        for t in self.tensors.values():
            _require(t.is_cuda and t.is_contiguous(), "weights must be contiguous CUDA tensors")
        hidden = attn_norm.numel()
        self.desc = _native.DecoderW8(
            hidden=hidden, heads=heads, head_dim=hidden // heads, ffn=w_down.shape[0],
            rms_eps=rms_eps, rope_theta=rope_theta,
            **{k: v.data_ptr() for k, v in self.tensors.items()})
        self._ws = None

    def workspace_bytes(self, batch: int, seq: int) -> int:
        import ctypes
        return _native.load().hxb_decoder_block_workspace_bytes(ctypes.byref(self.desc),
                                                                batch, seq)

    def __call__(self, x: torch.Tensor, *, batch: int = 1, pos0: int = 0,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        import ctypes
        lib = _native.load()
        rows = x.shape[0]
        seq = rows // batch
        need = self.workspace_bytes(batch, seq)
        _require(need > 0, "invalid decoder description")
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        if out is None:
            out = torch.empty_like(x)
        check(lib.hxb_decoder_block_w8a16(ctypes.byref(self.desc), x.data_ptr(), out.data_ptr(),
                                          batch, seq, pos0, self._ws.data_ptr(),
                                          self._ws.numel(), _stream_ptr(x)))
        return out

    def new_cache(self, batch: int, cache_rows: int, device=None) -> tuple[torch.Tensor, torch.Tensor]:
        """Zeroed K and V caches [batch, heads, cache_rows, head_dim] f16 (the
        registered buffers of the reference's SliceUpdateKvCache,
        integration_tests/models/kv_cache.py:91-99)."""
        d = self.desc
        shape = (batch, d.heads, cache_rows, d.head_dim)
        dev = device or self.tensors["w_qkv"].device
        return (torch.zeros(shape, dtype=torch.float16, device=dev),
                torch.zeros(shape, dtype=torch.float16, device=dev))

    def step(self, x: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *, pos0: int,
             batch: int = 1, out: torch.Tensor | None = None) -> torch.Tensor:
        """The block on x [batch * seq, hidden] at positions pos0 .. against a
        KV cache: writes the new rows' K/V into the caches and attends to
        cache rows [0, pos0 + seq) (hxb_decoder_block_w8a16_cached). A prompt
        at pos0 = 0 is the prefill; one row per batch at pos0 = tokens so far
        is a decode step."""
        import ctypes
        lib = _native.load()
        rows = x.shape[0]
        seq = rows // batch
        _require(k_cache.shape == v_cache.shape and k_cache.dim() == 4 and
                 k_cache.shape[0] == batch and k_cache.dtype == torch.float16 and
                 k_cache.is_contiguous() and v_cache.is_contiguous(),
                 "k_cache / v_cache must be contiguous f16 [batch, heads, rows, head_dim]")
        need = lib.hxb_decoder_block_cached_workspace_bytes(ctypes.byref(self.desc), batch, seq)
        _require(need > 0, "invalid decoder description")
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        if out is None:
            out = torch.empty_like(x)
        check(lib.hxb_decoder_block_w8a16_cached(
            ctypes.byref(self.desc), x.data_ptr(), out.data_ptr(), batch, seq, pos0,
            k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[2], self._ws.data_ptr(),
            self._ws.numel(), _stream_ptr(x)))
        return out


def kv_cache_write(k_src: torch.Tensor, v_src: torch.Tensor, k_cache: torch.Tensor,
                   v_cache: torch.Tensor, *, begin: int, batch: int = 1) -> None:
    """k_cache[b, h, begin + t] = k_src[b * n + t, h*D:(h+1)*D] (and V), the
    in-place cache update of SliceUpdateKvCache.update
    (integration_tests/models/kv_cache.py:101-112). Sources are [batch * n,
    >= heads * D] row-major views (unit inner stride), caches contiguous
    [batch, heads, rows, D] f16."""
    lib = _native.load()
    _require(k_cache.shape == v_cache.shape and k_cache.dim() == 4 and
             k_cache.is_contiguous() and v_cache.is_contiguous(), "bad cache tensors")
    _require(k_src.stride() == v_src.stride(), "k_src / v_src must share a layout")
    B, H, rows, D = k_cache.shape
    check(lib.hxb_kv_cache_write_f16(k_src.data_ptr(), v_src.data_ptr(), _rowmajor_ld(k_src, "k_src"),
                                     k_cache.data_ptr(), v_cache.data_ptr(), batch, H,
                                     k_src.shape[0] // batch, begin, rows, D, _stream_ptr(k_src)))


def device_status(clear: bool = True) -> int:
    """Status bits kernels raised on the current device (1 = a wait timed out)."""
    import ctypes
    bits = ctypes.c_int(0)
    check(_native.load().hxb_device_status(int(clear), ctypes.byref(bits)))
    return bits.value
