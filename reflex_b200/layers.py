"""Reflex layer modules on the rfx kernels: same names, constructor arguments,
methods and error behaviour as reflex/layers, so a Reflex policy can swap
them in behind ``enable_streaming`` / ``fuse_qkv`` / ``fuse_gate_up``.

* ``StreamingAttention``: reflex/layers/streaming_attention.py:91-637.  The
  source (prefix / observation-window) K/V live quantized in a static ring;
  decode attends to it directly with the partitioned attention kernel, so
  ``merge_caches`` only records the slice (no dequantize + copy) and
  ``split_caches`` is a no-op as in the reference's unified-buffer mode.
  ``quantize_kv_cache=True`` keeps the reference's uint8 scheme (bit-exact
  with its torch quantizer); ``quantize_kv_cache=False`` (the reference's
  default, which keeps a bf16 / fp16 source cache) stores the source as int8
  with one fp32 scale per token and head (absmax / 127), so each source value
  carries an error of at most absmax / 254 of its row.
* ``QKVLinear`` / ``MergedColumnLinear``: reflex/layers/linear.py:29-148, as
  ``nn.Module``s with ``nn.Parameter`` weights, so ``.to()``, ``state_dict``
  and the reference's fusion init (reflex/policies/pi05/modeling_pi05.py:
  843-866, 883-917) work on them unchanged.
* ``fused_quantize_store``: reflex/layers/quantize_kernel.py:58-79.

There is no CPU path: every method that computes needs CUDA tensors.
"""
from __future__ import annotations

import ctypes
import weakref

import torch
from torch import nn

from . import _lib as L
from . import kernels as K

_SCHEMES = {"u8_ref": L.RFX_QUANT_U8_REF, "i8_sym": L.RFX_QUANT_I8_SYM}


def fused_quantize_store(x: torch.Tensor, cache: torch.Tensor, scale: torch.Tensor, zp: torch.Tensor,
                         cache_start_idx: int = 0) -> None:
    """Quantizes x [B, H, L, D] per (b, h, token) into cache[:, :, start:start+L]
    (uint8) and scale / zp [B, H, cap, 1] (the activation dtype), with the
    interface of reflex/layers/quantize_kernel.py:58.  The arithmetic is the
    reference's torch quantizer (StreamingAttention._quantize,
    streaming_attention.py:211-218: range clamped at 1e-5, round half to
    even, every op in the activation dtype), bit-exact; the reference's Triton
    kernel differs from its own torch path on exact .5 ties (it rounds half
    up) and on ranges below 1e-6 (scale 1.0)."""
    if cache.dtype != torch.uint8 or cache.dim() != 4 or scale.shape[:3] != cache.shape[:3]:
        raise ValueError("cache must be uint8 [B, H, cap, D] with scale / zp [B, H, cap, 1]")
    if scale.dtype != x.dtype or zp.dtype != x.dtype:
        raise ValueError("scale and zero point are stored in the activation dtype")
    B, H, Lnew, D = x.shape
    if cache_start_idx < 0 or cache_start_idx + Lnew > cache.shape[2]:
        raise ValueError(f"cache_start_idx {cache_start_idx} + {Lnew} tokens exceeds the cache ({cache.shape[2]})")
    x = x.contiguous()
    d = L.KvQuantDesc()
    d.mode, d.in_dtype = L.RFX_QUANT_U8_REF, K._dtype_code(x)
    d.k, d.v = x.data_ptr(), None
    d.xs_b, d.xs_h, d.xs_l = x.stride(0), x.stride(1), x.stride(2)
    d.B, d.H, d.L, d.D = B, H, Lnew, D
    d.k_q, d.v_q = cache.data_ptr(), None
    d.qs_b, d.qs_h, d.qs_c = cache.stride(0), cache.stride(1), cache.stride(2)
    d.capacity = cache.shape[2]
    d.k_scale, d.v_scale = scale.data_ptr(), None
    d.k_zp, d.v_zp = zp.data_ptr(), None
    d.ss_b, d.ss_h, d.ss_c = scale.stride(0), scale.stride(1), scale.stride(2)
    d.region_base, d.region_off, d.region_len = 0, cache_start_idx, cache.shape[2]
    L.call("rfx_kv_quant_append", ctypes.byref(d), K._stream())


class StreamingAttention(nn.Module):
    """Streaming attention over a quantized source ring (see the module docstring).

    The source is a ring: logical source token i lives in slot
    (head + i) % max_cache_size, so ``evict_source_prefix`` moves the head in
    O(1) (the reference shift-copies the whole buffer) and appends wrap.  The
    attention kernel does not care about slot order: a slice of the source
    that wraps or starts past slot 0 is passed as a per-slot validity mask.

    ``kv_scheme`` overrides the scheme: "u8_ref" (the reference's uint8
    scheme, default with ``quantize_kv_cache=True``) or "i8_sym" (default with
    ``quantize_kv_cache=False``)."""

    def __init__(self, scale: float, enable_streaming: bool = True, block_size: int = 16,
                 use_blocked_cache: bool = False, max_cache_size: int = 2048, enable_flash_attention: bool = True,
                 enable_mixed_precision: bool = True, quantize_kv_cache: bool = False, *,
                 kv_scheme: str | None = None):
        super().__init__()
        if kv_scheme is None:
            kv_scheme = "u8_ref" if quantize_kv_cache else "i8_sym"
        if kv_scheme not in _SCHEMES:
            raise ValueError(f"kv_scheme must be one of {sorted(_SCHEMES)}")
        self.scale = scale
        self.enable_streaming = enable_streaming
        self.block_size = block_size
        self.use_blocked_cache = use_blocked_cache
        self.max_cache_size = max_cache_size
        self.enable_flash_attention = enable_flash_attention
        self.enable_mixed_precision = enable_mixed_precision
        self.quantize_kv_cache = quantize_kv_cache
        self.kv_scheme = kv_scheme
        self.ring: K.KVRing | None = None
        self.cache_stats = {"source_updates": 0, "source_tokens": 0, "attention_calls": 0, "mask_cache_hits": 0}
        self.reset_cache()

    # ------------------------------------------------------------- state ---
    def reset_cache(self, reset_stats: bool = False) -> None:
        self.ring = None
        self.source_length = 0
        self._head = 0  # slot of logical source token 0
        self._pending: list[tuple[torch.Tensor, torch.Tensor]] = []
        self._pending_source_length = 0
        self._merged: tuple[int, int] | None = None  # the merged source slice, once merge_caches ran
        self.merge_start_idx = 0
        self._struct_key = None
        self._struct_ref = None
        self._struct = None
        if reset_stats:
            self.cache_stats = {k: 0 for k in self.cache_stats}

    # reference attribute: callers test for merge support (modeling_pi05.py:804)
    @property
    def merged_k_cache(self):
        return self.ring.k_q if self._merged is not None and self.ring is not None else None

    def _init_ring(self, B: int, H: int, D: int, dtype: torch.dtype, device) -> None:
        mode = _SCHEMES[self.kv_scheme]
        sdt = dtype if mode == L.RFX_QUANT_U8_REF else torch.float32
        self.ring = K.KVRing.allocate(B, H, self.max_cache_size, D, mode, scale_dtype=sdt, device=device)

    def prefill_source(self, k: torch.Tensor, v: torch.Tensor, *, cache_slot: str = "main") -> None:
        """Appends source K/V [B, H, L, D] after the current source (quantized),
        or to the pending slot (committed later by commit_pending_source)."""
        if cache_slot not in ("main", "pending"):
            raise ValueError(f"cache_slot must be 'main' or 'pending', got {cache_slot}")
        if cache_slot == "pending":
            self._pending.append((k.detach(), v.detach()))
            self._pending_source_length += k.shape[2]
            return
        B, H, Lnew, D = k.shape
        if self.ring is None:
            self._init_ring(B, H, D, k.dtype, k.device)
        cap = self.ring.capacity
        if self.source_length + Lnew > cap:
            raise ValueError(f"source cache overflow: {self.source_length} + {Lnew} > max_cache_size "
                             f"{cap} (evict before appending)")
        K.kv_quant_append(k.contiguous(), v.contiguous(), self.ring, 0, (self._head + self.source_length) % cap, cap)
        self.source_length += Lnew
        self._struct_key = None
        self.cache_stats["source_updates"] += 1
        self.cache_stats["source_tokens"] += Lnew

    def commit_pending_source(self) -> None:
        if self._pending_source_length <= 0:
            return
        k = torch.cat([p[0] for p in self._pending], dim=2)
        v = torch.cat([p[1] for p in self._pending], dim=2)
        self._pending, self._pending_source_length = [], 0
        self.prefill_source(k, v, cache_slot="main")

    def evict_source_prefix(self, num_tokens: int) -> None:
        """Drops the oldest num_tokens source tokens: the ring head moves past
        them (no data is copied)."""
        if num_tokens <= 0 or self.source_length <= 0 or self.ring is None:
            return
        n = min(int(num_tokens), int(self.source_length))
        self._head = (self._head + n) % self.ring.capacity
        self.source_length -= n
        self._struct_key = None

    def merge_caches(self, source_start_idx: int = 0, source_end_idx: int | None = None) -> None:
        """Selects the source slice the next decode attends to."""
        if self.ring is None or self.source_length == 0:
            self._merged = None
            return
        end = self.source_length if source_end_idx is None else int(source_end_idx)
        start = int(source_start_idx)
        if not 0 <= start <= end <= self.source_length:
            raise ValueError(f"source slice [{start}, {end}) outside [0, {self.source_length})")
        self._merged = (start, end)
        self.merge_start_idx = start

    def split_caches(self) -> None:
        pass

    def source_slots(self, start: int, end: int, device=None) -> torch.Tensor:
        """Ring slots of the logical source tokens [start, end)."""
        return (self._head + torch.arange(start, end, device=device)) % self.ring.capacity

    # ------------------------------------------------------------ decode ---
    @staticmethod
    def _mask_to_structure(mask: torch.Tensor, B: int, Lq: int, n_src: int, src_start: int):
        """A boolean / additive mask [B, 1, Lq, n_src + Lq] whose source part
        is the same for every query row and whose suffix part is
        block-causal -> (per-stream validity of logical source tokens
        [0, src_start + n_src), suffix block ids).  Anything else raises
        ValueError."""
        allow = mask if mask.dtype == torch.bool else mask == 0
        allow = allow.reshape(B, -1, Lq, allow.shape[-1])[:, 0]
        if allow.shape[-1] != n_src + Lq:
            raise ValueError(f"attention_mask has {allow.shape[-1]} keys, expected {n_src + Lq}")
        src = allow[:, :, :n_src]
        if not bool((src == src[:, :1]).all()):
            raise ValueError("attention_mask: every query row must see the same source tokens")
        suf = allow[0, :, n_src:]
        if not bool((allow[:, :, n_src:] == suf).all()):
            raise ValueError("attention_mask: the suffix pattern must be the same for every stream")
        # query row i is in block rank(count of keys it sees); key j is in the
        # lowest block of the rows that see it; block-causal means row i sees
        # exactly the keys of blocks <= its own, and every token's key and
        # query blocks agree
        counts = suf.sum(dim=1)
        levels = torch.unique(counts, sorted=True)
        block = torch.searchsorted(levels, counts).to(torch.int32)
        big = torch.full_like(block, int(levels.numel()))
        key_block = torch.where(suf, block[:, None], big[:, None]).min(dim=0).values
        rebuilt = key_block[None, :] <= block[:, None]
        if not torch.equal(rebuilt, suf) or not torch.equal(key_block, block):
            raise ValueError("attention_mask: the suffix part is not block-causal")
        valid = torch.zeros(B, src_start + n_src, dtype=torch.uint8, device=mask.device)
        valid[:, src_start:] = src[:, 0].to(torch.uint8)
        return valid, block

    def _structure(self, mask: torch.Tensor | None, B: int, Lq: int, start: int, end: int, device):
        """(n_ctx, ctx_valid, new_block) of a decode, cached: the 18 layers of a
        denoising step get the same mask tensor, so only the first layer that
        sees a mask checks it (the checks read it back to the host); a mask
        modified in place, another mask object, or a change of the source
        (append, evict, slice) recomputes it."""
        key = (id(mask) if mask is not None else None, mask._version if mask is not None else None,
               tuple(mask.shape) if mask is not None else None, B, Lq, start, end, self._head, self.source_length)
        if (self._struct_key == key and
                (mask is None or (self._struct_ref is not None and self._struct_ref() is mask))):
            self.cache_stats["mask_cache_hits"] += 1
            return self._struct
        n_src = end - start
        new_block = None
        valid = None
        if mask is not None:
            valid, block = self._mask_to_structure(mask, B, Lq, n_src, start)
            new_block = block.contiguous()
            if n_src and bool(valid[:, start:end].all()):
                valid = None  # every source token of the slice is visible
        cap = self.ring.capacity if self.ring is not None else 0
        if n_src == 0:
            struct = (0, None, new_block)
        elif valid is None and self._head + start == 0:
            struct = (n_src, None, new_block)  # the slice is slots [0, n_src)
        else:
            ctx_valid = torch.zeros(B, cap, dtype=torch.uint8, device=device)
            slots = self.source_slots(start, end, device)
            ctx_valid[:, slots] = valid[:, start:end] if valid is not None else 1
            struct = (cap, ctx_valid, new_block)
        self._struct_key = key
        self._struct_ref = weakref.ref(mask) if mask is not None else None
        self._struct = struct
        return struct

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attention_mask: torch.Tensor | None = None,
                use_cache: bool = False, is_prefix: bool = False, is_suffix: bool = False, cache_slot: str = "main",
                merge_before_decode: bool = False, source_slice_start: int = 0, source_slice_end: int | None = None,
                split_after_decode: bool = False) -> torch.Tensor:
        """q [B, Hq, Lq, 256] bf16, k / v [B, 1, Lq, 256] -> [B, Hq, Lq, 256]."""
        if use_cache and is_prefix:
            self.prefill_source(k, v, cache_slot=cache_slot)
            return torch.zeros_like(q)
        if merge_before_decode:
            self.merge_caches(source_slice_start, source_slice_end)
        B, Hq, Lq, D = q.shape
        if k.shape[1] != 1:
            raise ValueError("the attention kernel serves one shared KV head (MQA)")
        start, end = self._merged if self._merged is not None else (0, 0)
        n_ctx, ctx_valid, new_block = self._structure(attention_mask, B, Lq, start, end, q.device)
        out = torch.empty(B * Lq, Hq * D, dtype=torch.bfloat16, device=q.device)
        qc = q.to(torch.bfloat16).contiguous()
        ks = k[:, 0].to(torch.bfloat16).contiguous()
        vs = v[:, 0].to(torch.bfloat16).contiguous()
        K.attention(q=qc, k_new=ks, v_new=vs, ring=self.ring if n_ctx else None, n_ctx=n_ctx,
                    out=out, softmax_scale=self.scale, ctx_valid=ctx_valid, new_block=new_block)
        self.cache_stats["attention_calls"] += 1
        if split_after_decode:
            self.split_caches()
        return out.view(B, Lq, Hq, D).transpose(1, 2)


class _RfxLinear(nn.Module):
    """Shared part of the fused projections: a bf16 copy of the parameters
    for the kernel, refreshed when the weight or bias changes (their
    ``_version`` counts in-place writes, as the reference's fusion init makes)."""

    def _kernel_operands(self):
        w, b = self.weight, self.bias
        key = (w.data_ptr(), w._version, w.dtype, w.device, None if b is None else (b.data_ptr(), b._version))
        if getattr(self, "_op_key", None) != key:
            with torch.no_grad():
                wk = w.detach().to(torch.bfloat16).contiguous()
                bk = b.detach().to(torch.float32).contiguous() if b is not None else None
            self._ops = (wk, bk)
            self._op_key = key
        return self._ops

    def _project(self, x2: torch.Tensor, T: int, S: int) -> torch.Tensor:
        if not x2.is_cuda or not self.weight.is_cuda:
            raise ValueError(f"{type(self).__name__} runs on the rfx kernels: move the module and input to CUDA")
        wk, bk = self._kernel_operands()
        y = torch.empty(T, wk.shape[0], dtype=torch.bfloat16, device=x2.device)
        K.linear(w=wk, x=x2.to(torch.bfloat16).contiguous(), T=T, S=S, epilogue=L.RFX_EPI_STORE, bias=bk, y=y)
        return y


class QKVLinear(_RfxLinear):
    """Fused [Wq; Wk; Wv] projection (reflex/layers/linear.py:29-98):
    forward(x [B, L, hidden]) -> (q [B, H, L, D], k [B, Hkv, L, D], v [B, Hkv, L, D]).
    The product runs in bf16 with fp32 accumulation; outputs come back in the
    input's dtype, as F.linear's would."""

    def __init__(self, hidden_size: int, head_size: int, total_num_heads: int, total_num_kv_heads: int | None = None,
                 bias: bool = False):
        super().__init__()
        total_num_kv_heads = total_num_kv_heads or total_num_heads
        self.hidden_size, self.head_size = hidden_size, head_size
        self.num_heads, self.num_kv_heads = total_num_heads, total_num_kv_heads
        rows = (self.num_heads + 2 * self.num_kv_heads) * head_size
        self.weight = nn.Parameter(torch.empty(rows, hidden_size))
        if bias:
            self.bias = nn.Parameter(torch.empty(rows))
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor):
        if x.dim() != 3:
            raise ValueError(f"QKVLinear expects 3D input [B, L, D], got {x.shape}")
        B, Lx, Hd = x.shape
        y = self._project(x.reshape(B * Lx, Hd), B * Lx, Lx).to(x.dtype)
        D, H, Hk = self.head_size, self.num_heads, self.num_kv_heads
        q = y[:, :H * D].view(B, Lx, H, D).transpose(1, 2)
        k = y[:, H * D:(H + Hk) * D].view(B, Lx, Hk, D).transpose(1, 2)
        v = y[:, (H + Hk) * D:].view(B, Lx, Hk, D).transpose(1, 2)
        return q, k, v


class MergedColumnLinear(_RfxLinear):
    """Column-merged projection (reflex/layers/linear.py:103-148):
    forward(x [..., in]) -> tuple of [..., output_sizes[i]] (bf16 product,
    fp32 accumulation, outputs in the input's dtype)."""

    def __init__(self, input_size: int, output_sizes: list[int], bias: bool = False):
        super().__init__()
        self.input_size, self.output_sizes = input_size, list(output_sizes)
        out = sum(self.output_sizes)
        self.weight = nn.Parameter(torch.empty(out, input_size))
        if bias:
            self.bias = nn.Parameter(torch.empty(out))
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor):
        shape = x.shape[:-1]
        T = 1
        for s in shape:
            T *= int(s)
        y = self._project(x.reshape(T, self.input_size), T, T).to(x.dtype)
        return tuple(t.reshape(*shape, t.shape[-1]) for t in torch.split(y, self.output_sizes, dim=-1))
