"""Thin torch-tensor wrappers over the librfx_b200 C ABI.

Each function validates dtypes/devices, fills the descriptor declared in
include/rfx.h and calls the library on the current CUDA stream.  Tensors must
live on a CUDA device: there is no CPU path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("rfx kernels take CUDA tensors only (there is no CPU fallback)")


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return L.RFX_DTYPE_BF16
    if t.dtype == torch.float32:
        return L.RFX_DTYPE_F32
    raise ValueError(f"unsupported dtype {t.dtype}")


# --------------------------------------------------------------- KV ring ---
@dataclass
class KVRing:
    """Quantized KV storage of one attention layer: [B, H, capacity, D] payload
    plus per-slot scales (and zero points in the reference uint8 scheme)."""

    k_q: torch.Tensor
    v_q: torch.Tensor
    k_scale: torch.Tensor
    v_scale: torch.Tensor
    k_zp: torch.Tensor | None
    v_zp: torch.Tensor | None
    mode: int

    @staticmethod
    def allocate(B: int, H: int, capacity: int, D: int, mode: int, scale_dtype=torch.bfloat16,
                 device="cuda") -> "KVRing":
        qdt = torch.int8 if mode == L.RFX_QUANT_I8_SYM else torch.uint8
        sdt = torch.float32 if mode == L.RFX_QUANT_I8_SYM else scale_dtype
        mk = lambda shape, dt: torch.zeros(shape, dtype=dt, device=device)  # noqa: E731
        zp = (lambda: mk((B, H, capacity), sdt)) if mode == L.RFX_QUANT_U8_REF else (lambda: None)
        return KVRing(mk((B, H, capacity, D), qdt), mk((B, H, capacity, D), qdt),
                      mk((B, H, capacity), sdt), mk((B, H, capacity), sdt), zp(), zp(), mode)

    @property
    def capacity(self) -> int:
        return self.k_q.shape[2]


def kv_quant_desc(k: torch.Tensor, v: torch.Tensor, ring: KVRing, region_base: int, region_off: int,
                  region_len: int) -> L.KvQuantDesc:
    _need_cuda(k, v, ring.k_q)
    if k.shape != v.shape or k.dim() != 4 or k.stride(-1) != 1 or v.stride() != k.stride():
        raise ValueError("k/v must be [B, H, L, D] with matching strides and contiguous D")
    if ring.k_scale.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("ring scale dtype")
    if ring.mode == L.RFX_QUANT_U8_REF and ring.k_scale.dtype != k.dtype:
        raise ValueError("reference uint8 scheme stores scale/zp in the activation dtype")
    B, H, Lnew, D = k.shape
    d = L.KvQuantDesc()
    d.mode, d.in_dtype = ring.mode, _dtype_code(k)
    d.k, d.v = k.data_ptr(), v.data_ptr()
    d.xs_b, d.xs_h, d.xs_l = k.stride(0), k.stride(1), k.stride(2)
    d.B, d.H, d.L, d.D = B, H, Lnew, D
    d.k_q, d.v_q = ring.k_q.data_ptr(), ring.v_q.data_ptr()
    d.qs_b, d.qs_h, d.qs_c = ring.k_q.stride(0), ring.k_q.stride(1), ring.k_q.stride(2)
    d.capacity = ring.capacity
    d.k_scale, d.v_scale = ring.k_scale.data_ptr(), ring.v_scale.data_ptr()
    d.k_zp = ring.k_zp.data_ptr() if ring.k_zp is not None else None
    d.v_zp = ring.v_zp.data_ptr() if ring.v_zp is not None else None
    d.ss_b, d.ss_h, d.ss_c = ring.k_scale.stride(0), ring.k_scale.stride(1), ring.k_scale.stride(2)
    d.region_base, d.region_off, d.region_len = region_base, region_off, region_len
    return d


def kv_quant_append(k, v, ring: KVRing, region_base: int = 0, region_off: int = 0, region_len: int | None = None):
    """Quantizes k/v [B,H,L,D] into ring slots region_base + (region_off + l) % region_len."""
    if region_len is None:
        region_len = ring.capacity - region_base
    d = kv_quant_desc(k, v, ring, region_base, region_off, region_len)
    L.call("rfx_kv_quant_append", ctypes.byref(d), _stream())


# ---------------------------------------------------------------- linear ---
def pack_weight(kind: int, w: torch.Tensor) -> torch.Tensor:
    _need_cuda(w)
    if w.dtype != torch.bfloat16 or not w.is_contiguous():
        raise ValueError("pack_weight takes a contiguous bf16 [rows, K] weight")
    out = torch.empty_like(w)
    L.call("rfx_pack_weight", kind, w.data_ptr(), out.data_ptr(), w.shape[0], w.shape[1], _stream())
    return out


def linear_desc(*, w, x, T, S, prologue=L.RFX_PRO_LOAD, epilogue=L.RFX_EPI_STORE, y=None, norm_a1=None,
                norm_a2=None, norm_b2=None, norm_ab_stride=0, eps=1e-6, bias=None, gate=None, gate_stride=0,
                rope_table=None, positions=None, q_out=None, k_out=None, v_out=None, num_q_heads=0,
                n_tile=0, splits=0, y_rows_per_batch=0, y_row_offset=0,
                workspace=None) -> L.LinearDesc:
    _need_cuda(w, x, y)
    for t in (w, x, y, q_out, k_out, v_out):
        if t is not None and t.dtype != torch.bfloat16:
            raise ValueError("linear operands are bf16")
    for t in (norm_a1, norm_a2, norm_b2, bias, gate, rope_table):
        if t is not None and t.dtype != torch.float32:
            raise ValueError("norm/bias/gate/rope vectors are fp32")
    d = L.LinearDesc()
    d.T, d.O, d.K, d.tokens_per_batch = T, w.shape[0], w.shape[1], S
    d.prologue, d.epilogue = prologue, epilogue
    d.w, d.x, d.ldx = w.data_ptr(), x.data_ptr(), x.stride(0)
    d.norm_a1, d.norm_a2, d.norm_b2 = L.ptr(norm_a1), L.ptr(norm_a2), L.ptr(norm_b2)
    d.norm_ab_stride, d.eps = norm_ab_stride, eps
    d.y = L.ptr(y)
    d.ldy = y.stride(0) if y is not None else 0
    d.bias, d.gate, d.gate_stride = L.ptr(bias), L.ptr(gate), gate_stride
    d.rope_table = L.ptr(rope_table)
    d.rope_max_pos = rope_table.shape[0] if rope_table is not None else 0
    if positions is not None and positions.dtype != torch.int32:
        raise ValueError("positions are int32")
    d.positions = L.ptr(positions)
    d.q_out, d.k_out, d.v_out = L.ptr(q_out), L.ptr(k_out), L.ptr(v_out)
    d.num_q_heads = num_q_heads
    d.n_tile, d.splits = n_tile, splits
    d.y_rows_per_batch, d.y_row_offset = y_rows_per_batch, y_row_offset
    d.workspace = L.ptr(workspace)
    d.workspace_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    return d


def linear(**kw) -> None:
    d = linear_desc(**kw)
    L.call("rfx_linear", ctypes.byref(d), _stream())


def linear_workspace_bytes(d: L.LinearDesc) -> int:
    """Split-K workspace rfx_linear would use for `d` (0: none)."""
    n = ctypes.c_size_t(0)
    L.call("rfx_linear_workspace_size", ctypes.byref(d), ctypes.byref(n))
    return n.value


def linear_workspace(nbytes: int, device) -> torch.Tensor:
    """A zero-filled split-K workspace (the counters start at zero); pass
    aligned_ptr(ws, 256) or a 256-byte aligned slice of it."""
    return torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=device)


# ------------------------------------------------------------- attention ---
def attention_desc(*, q, k_new, v_new, ring: KVRing | None, n_ctx: int, out, softmax_scale: float,
                   workspace=None, ctx_valid=None, new_block=None, kv_splits=0,
                   kv_source: int = L.RFX_KV_RING_TILES) -> L.AttnDesc:
    _need_cuda(q, k_new, v_new, out)
    B, Hq, S, D = q.shape
    d = L.AttnDesc()
    d.B, d.num_q_heads, d.head_dim, d.S = B, Hq, D, S
    d.capacity = ring.capacity if ring is not None else 0
    d.n_ctx = n_ctx
    d.quant_mode = ring.mode if ring is not None else L.RFX_QUANT_I8_SYM
    d.scale_dtype = _dtype_code(ring.k_scale) if ring is not None else L.RFX_DTYPE_F32
    d.q, d.k_new, d.v_new = q.data_ptr(), k_new.data_ptr(), v_new.data_ptr()
    if ring is not None:
        if ring.k_q.shape[1] != 1:
            raise ValueError("the attention kernel serves one shared KV head (MQA)")
        d.k_ring, d.v_ring = ring.k_q.data_ptr(), ring.v_q.data_ptr()
        d.k_scale, d.v_scale = ring.k_scale.data_ptr(), ring.v_scale.data_ptr()
        d.k_zp, d.v_zp = L.ptr(ring.k_zp), L.ptr(ring.v_zp)
    d.ctx_valid, d.new_block = L.ptr(ctx_valid), L.ptr(new_block)
    d.softmax_scale = softmax_scale
    d.out = out.data_ptr()
    d.workspace = L.ptr(workspace)
    d.workspace_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    d.kv_splits = kv_splits
    d.kv_source = kv_source
    return d


def attention_workspace_bytes(d: L.AttnDesc) -> int:
    n = ctypes.c_size_t(0)
    L.call("rfx_attention_workspace_size", ctypes.byref(d), ctypes.byref(n))
    return n.value


def attention(**kw) -> None:
    """Partitioned attention; allocates the split-KV workspace if the caller did not."""
    d = attention_desc(**kw)
    need = attention_workspace_bytes(d)
    ws = kw.get("workspace")
    if need and (ws is None or ws.numel() * ws.element_size() < need or ws.data_ptr() % 1024):
        ws = torch.zeros(need + 1024, dtype=torch.uint8, device=kw["q"].device)
        d.workspace, d.workspace_bytes = aligned_ptr(ws, 1024), need
    L.call("rfx_attention", ctypes.byref(d), _stream())


def aligned_ptr(buf: torch.Tensor, align: int) -> int:
    """First `align`-byte aligned address inside `buf` (allocate `align` spare bytes)."""
    return (buf.data_ptr() + align - 1) // align * align


# ----------------------------------------------------- conditioning heads ---
def time_cond_desc(*, t, w_in, b_in, w_out, b_out, hidden, cond, min_period, max_period) -> L.TimeCondDesc:
    """w_in = None computes the bf16 sinusoidal embedding alone (into `cond`)."""
    _need_cuda(t, w_in, cond)
    d = L.TimeCondDesc()
    d.n_t, d.t, d.width = t.numel(), t.data_ptr(), cond.shape[1]
    d.min_period, d.max_period = min_period, max_period
    d.w_in, d.b_in, d.w_out, d.b_out = L.ptr(w_in), L.ptr(b_in), L.ptr(w_out), L.ptr(b_out)
    d.hidden, d.cond = L.ptr(hidden), cond.data_ptr()
    return d


def time_cond(**kw) -> None:
    d = time_cond_desc(**kw)
    L.call("rfx_time_cond", ctypes.byref(d), _stream())


def modulation_desc(*, mode, w, b, cond, a2, b2, gate, n_norms) -> L.ModulationDesc:
    _need_cuda(w, cond, a2)
    d = L.ModulationDesc()
    d.mode, d.n_rows, d.n_norms, d.width = mode, cond.shape[0], n_norms, cond.shape[1]
    d.w, d.b, d.cond = w.data_ptr(), b.data_ptr(), cond.data_ptr()
    d.a2, d.b2, d.gate = a2.data_ptr(), L.ptr(b2), gate.data_ptr()
    return d


def modulation(**kw) -> None:
    d = modulation_desc(**kw)
    L.call("rfx_modulation", ctypes.byref(d), _stream())


def action_io_desc(*, B, S, S_total, x, w_in, b_in, h_next=None, h_next_rows_per_stream=None,
                   h_next_row_offset=0, h=None, h_row_offset=0, norm_a1=None, norm_a2=None, norm_b2=None,
                   norm_ab_stride=0, eps=1e-6, w_out=None, b_out=None, dt=0.0) -> L.ActionIoDesc:
    _need_cuda(x, w_in, h, h_next)
    d = L.ActionIoDesc()
    d.B, d.S, d.S_total, d.action_dim = B, S, S_total, x.shape[-1]
    d.width = w_in.shape[0]
    d.h_row_offset, d.h = h_row_offset, L.ptr(h)
    d.norm_a1, d.norm_a2, d.norm_b2 = L.ptr(norm_a1), L.ptr(norm_a2), L.ptr(norm_b2)
    d.norm_ab_stride, d.eps = norm_ab_stride, eps
    d.w_out, d.b_out, d.x, d.dt = L.ptr(w_out), L.ptr(b_out), x.data_ptr(), dt
    d.w_in, d.b_in = w_in.data_ptr(), L.ptr(b_in)
    d.h_next = L.ptr(h_next)
    d.h_next_ld = h_next.stride(0) if h_next is not None else 0
    d.h_next_rows_per_stream = h_next_rows_per_stream if h_next_rows_per_stream is not None else S_total
    d.h_next_row_offset = h_next_row_offset
    return d


def action_in(**kw) -> None:
    d = action_io_desc(**kw)
    L.call("rfx_action_in", ctypes.byref(d), _stream())


def euler_tail(**kw) -> None:
    d = action_io_desc(**kw)
    L.call("rfx_euler_tail", ctypes.byref(d), _stream())


def norm_desc(*, x, y, S, norm_a1, norm_a2=None, norm_b2=None, norm_ab_stride=0, eps=1e-6, T=None) -> L.NormDesc:
    _need_cuda(x, y, norm_a1)
    if x.dtype != torch.bfloat16 or y.dtype != torch.bfloat16:
        raise ValueError("rms_norm maps bf16 rows to bf16 rows")
    for t in (norm_a1, norm_a2, norm_b2):
        if t is not None and t.dtype != torch.float32:
            raise ValueError("norm vectors are fp32")
    d = L.NormDesc()
    d.T = x.shape[0] if T is None else T
    d.K, d.tokens_per_batch = x.shape[1], S
    d.x, d.ldx = x.data_ptr(), x.stride(0)
    d.norm_a1, d.norm_a2, d.norm_b2 = L.ptr(norm_a1), L.ptr(norm_a2), L.ptr(norm_b2)
    d.norm_ab_stride, d.eps = norm_ab_stride, eps
    d.y, d.ldy = y.data_ptr(), y.stride(0)
    return d


def rms_norm(**kw) -> None:
    d = norm_desc(**kw)
    L.call("rfx_rms_norm", ctypes.byref(d), _stream())


def patches_desc(*, image, out, patch) -> L.PatchesDesc:
    """Patch rows of [B, C, H, W] fp32 images for the patch convolution as a GEMM."""
    _need_cuda(image, out)
    if image.dtype != torch.float32 or out.dtype != torch.bfloat16 or not image.is_contiguous():
        raise ValueError("patches: contiguous fp32 images -> bf16 rows")
    d = L.PatchesDesc()
    d.B, d.C, d.H, d.W = image.shape
    d.patch = patch
    d.image, d.out, d.ldo = image.data_ptr(), out.data_ptr(), out.stride(0)
    return d


def layer_norm_desc(*, x, y, w, b, eps=1e-6, T=None) -> L.LayerNormDesc:
    _need_cuda(x, y, w, b)
    if x.dtype != torch.bfloat16 or y.dtype != torch.bfloat16 or w.dtype != torch.float32 or b.dtype != torch.float32:
        raise ValueError("layer_norm maps bf16 rows to bf16 rows with fp32 weight and bias")
    d = L.LayerNormDesc()
    d.T = x.shape[0] if T is None else T
    d.C = x.shape[1]
    d.x, d.ldx = x.data_ptr(), x.stride(0)
    d.w, d.b, d.eps = w.data_ptr(), b.data_ptr(), eps
    d.y, d.ldy = y.data_ptr(), y.stride(0)
    return d


def vit_attention_desc(*, qkv, out, B, N, H, D, scale) -> L.VitAttnDesc:
    _need_cuda(qkv, out)
    if qkv.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise ValueError("vit_attention: bf16 q|k|v rows -> bf16 rows")
    d = L.VitAttnDesc()
    d.B, d.N, d.H, d.D = B, N, H, D
    d.qkv, d.ld_qkv = qkv.data_ptr(), qkv.stride(0)
    d.out, d.ld_out = out.data_ptr(), out.stride(0)
    d.scale = scale
    return d


def copy_rows_desc(*, dst, src, rows, width, dst_rows_per_group, dst_row_offset=0, group=None,
                   src_ld=None) -> L.CopyRowsDesc:
    _need_cuda(dst, src)
    if dst.dtype != torch.bfloat16 or src.dtype != torch.bfloat16:
        raise ValueError("copy_rows moves bf16 rows")
    d = L.CopyRowsDesc()
    d.dst, d.dst_ld = dst.data_ptr(), dst.stride(0)
    d.dst_rows_per_group, d.dst_row_offset = dst_rows_per_group, dst_row_offset
    d.group = group if group is not None else dst_rows_per_group
    d.src = src.data_ptr()
    d.src_ld = src.stride(0) if src_ld is None else src_ld
    d.rows, d.width = rows, width
    return d


def copy_rows(**kw) -> None:
    d = copy_rows_desc(**kw)
    L.call("rfx_copy_rows", ctypes.byref(d), _stream())


def device_status() -> int:
    v = ctypes.c_int(0)
    L.call("rfx_device_status", _stream(), ctypes.byref(v))
    return v.value


# ------------------------------------------------------------------ plans ---
class Plan:
    """Native ordered launch list (rfx_plan) with optional CUDA-graph capture."""

    _ADD = {
        L.LinearDesc: "rfx_plan_add_linear",
        L.AttnDesc: "rfx_plan_add_attention",
        L.KvQuantDesc: "rfx_plan_add_kv_quant",
        L.TimeCondDesc: "rfx_plan_add_time_cond",
        L.ModulationDesc: "rfx_plan_add_modulation",
        L.CopyRowsDesc: "rfx_plan_add_copy_rows",
        L.NormDesc: "rfx_plan_add_rms_norm",
        L.PatchesDesc: "rfx_plan_add_patches",
        L.LayerNormDesc: "rfx_plan_add_layer_norm",
        L.VitAttnDesc: "rfx_plan_add_vit_attention",
    }
    # direct (non-plan) entry point of each descriptor kind, for eager execution
    DIRECT = {
        L.LinearDesc: "rfx_linear",
        L.AttnDesc: "rfx_attention",
        L.KvQuantDesc: "rfx_kv_quant_append",
        L.TimeCondDesc: "rfx_time_cond",
        L.ModulationDesc: "rfx_modulation",
        L.CopyRowsDesc: "rfx_copy_rows",
        L.NormDesc: "rfx_rms_norm",
        L.PatchesDesc: "rfx_patches",
        L.LayerNormDesc: "rfx_layer_norm",
        L.VitAttnDesc: "rfx_vit_attention",
    }

    @classmethod
    def run_direct(cls, desc, kind: str | None = None) -> None:
        """Runs one descriptor through its direct C entry point on the current stream."""
        name = cls.DIRECT.get(type(desc))
        if isinstance(desc, L.ActionIoDesc):
            name = {"in": "rfx_action_in", "tail": "rfx_euler_tail"}[kind]
        L.call(name, ctypes.byref(desc), _stream())

    def __init__(self):
        self._h = ctypes.c_void_p()
        L.call("rfx_plan_create", ctypes.byref(self._h))
        self.captured = False

    def add(self, desc, kind: str | None = None) -> None:
        if kind == "barrier":
            L.call("rfx_plan_add_barrier", self._h)
            return
        if kind == "chunk":  # desc is an rfx_chunk handle
            L.call("rfx_plan_add_chunk", self._h, desc)
            return
        name = self._ADD.get(type(desc))
        if isinstance(desc, L.ActionIoDesc):
            name = {"in": "rfx_plan_add_action_in", "tail": "rfx_plan_add_euler_tail"}[kind]
        L.call(name, self._h, ctypes.byref(desc))

    @property
    def num_launches(self) -> int:
        n = ctypes.c_int(0)
        L.call("rfx_plan_num_launches", self._h, ctypes.byref(n))
        return n.value

    def run(self) -> None:
        L.call("rfx_plan_run", self._h, _stream())

    def capture(self, stream: torch.cuda.Stream) -> None:
        L.call("rfx_plan_capture", self._h, stream.cuda_stream)
        self.captured = True

    def replay(self) -> None:
        L.call("rfx_plan_replay", self._h, _stream())

    def close(self) -> None:
        if self._h:
            L.load().rfx_plan_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
