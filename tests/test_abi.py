"""The C ABI without a GPU: the library loads, exports every function that
include/rfx.h declares, the ctypes mirror matches the C struct layouts
(checked by compiling the header with gcc), and argument checks that need no
device return RFX_E_INVAL.
"""
import ctypes
import os
import re
import subprocess

import pytest

from reflex_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rfx.h")

STRUCTS = {
    "rfx_kv_quant_desc": "KvQuantDesc", "rfx_linear_desc": "LinearDesc", "rfx_norm_desc": "NormDesc",
    "rfx_attn_desc": "AttnDesc", "rfx_time_cond_desc": "TimeCondDesc", "rfx_modulation_desc": "ModulationDesc",
    "rfx_action_io_desc": "ActionIoDesc", "rfx_copy_rows_desc": "CopyRowsDesc", "rfx_chunk_desc": "ChunkDesc",
    "rfx_embed_cache_desc": "EmbedCacheDesc", "rfx_patches_desc": "PatchesDesc",
    "rfx_layer_norm_desc": "LayerNormDesc", "rfx_vit_attn_desc": "VitAttnDesc",
}


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_]+\s*\**\s*(rfx_[a-z0-9_]+)\s*\(", src, flags=re.M)))


def test_library_exports_every_declared_function():
    lib = _lib.load()
    names = header_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert sorted(_lib.SIGNATURES) == names, "ctypes signatures and header disagree"
    assert lib.rfx_version() >= 100


def test_ctypes_structs_match_c_layout(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "rfx.h"', "int main(void) {"]
    for c_name, py_name in STRUCTS.items():
        lines.append(f'  printf("{py_name} size %zu\\n", sizeof({c_name}));')
        for field, _ in getattr(_lib, py_name)._fields_:
            lines.append(f'  printf("{py_name} {field} %zu\\n", offsetof({c_name}, {field}));')
    lines.append("  return 0; }")
    c = tmp_path / "layout.c"
    c.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.dirname(HEADER), str(c), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    for line in filter(None, out):
        py_name, key, val = line.split()
        cls = getattr(_lib, py_name)
        got = ctypes.sizeof(cls) if key == "size" else getattr(cls, key).offset
        assert got == int(val), f"{py_name}.{key}: ctypes {got}, C {val}"


@pytest.mark.parametrize("name", ["rfx_linear", "rfx_attention", "rfx_attention_noalloc", "rfx_kv_quant_append",
                                  "rfx_rms_norm", "rfx_time_cond", "rfx_modulation", "rfx_action_in",
                                  "rfx_euler_tail", "rfx_copy_rows"])
def test_null_descriptor_is_rejected(name):
    lib = _lib.load()
    rc = getattr(lib, name)(None, None)
    assert rc == _lib.RFX_E_INVAL
    assert lib.rfx_last_error()


def test_plan_calls_out_of_order():
    lib = _lib.load()
    plan = ctypes.c_void_p()
    assert lib.rfx_plan_create(ctypes.byref(plan)) == _lib.RFX_OK
    try:
        assert lib.rfx_plan_replay(plan, None) == _lib.RFX_E_STATE
        n = ctypes.c_int(-1)
        assert lib.rfx_plan_num_launches(plan, ctypes.byref(n)) == _lib.RFX_OK and n.value == 0
    finally:
        assert lib.rfx_plan_destroy(plan) == _lib.RFX_OK


def test_plan_adds_check_descriptors():
    """Every plan add runs its op's descriptor check when the op is added (no
    device needed for the ops without tensor maps): a bad descriptor is
    refused with RFX_E_INVAL and leaves the plan as it was; good ones are
    counted by their launches (time conditioning with its MLP: three)."""
    lib = _lib.load()
    plan = ctypes.c_void_p()
    assert lib.rfx_plan_create(ctypes.byref(plan)) == _lib.RFX_OK
    n = ctypes.c_int(-1)
    try:
        norm = _lib.NormDesc()
        norm.T, norm.K, norm.tokens_per_batch = 50, 1024, 50
        norm.x = norm.y = norm.norm_a1 = 1 << 20  # aligned, never dereferenced
        norm.ldx = norm.ldy = 1024
        assert lib.rfx_plan_add_rms_norm(plan, ctypes.byref(norm)) == _lib.RFX_OK
        norm.K = norm.ldx = norm.ldy = 1020  # K % 8 != 0
        assert lib.rfx_plan_add_rms_norm(plan, ctypes.byref(norm)) == _lib.RFX_E_INVAL
        assert b"rfx_rms_norm" in lib.rfx_last_error()

        cp = _lib.CopyRowsDesc()
        cp.dst = cp.src = 1 << 20
        cp.rows, cp.width, cp.group, cp.dst_rows_per_group, cp.dst_row_offset = 50, 1024, 50, 51, 1
        cp.dst_ld = cp.src_ld = 1024
        assert lib.rfx_plan_add_copy_rows(plan, ctypes.byref(cp)) == _lib.RFX_OK
        cp.dst_row_offset = 2  # group of 50 from row 2 overruns 51 rows
        assert lib.rfx_plan_add_copy_rows(plan, ctypes.byref(cp)) == _lib.RFX_E_INVAL

        tc = _lib.TimeCondDesc()
        tc.n_t, tc.width, tc.min_period, tc.max_period = 10, 1024, 4e-3, 4.0
        tc.t = 1 << 20
        tc.w_in = tc.b_in = tc.w_out = tc.b_out = tc.hidden = tc.cond = 1 << 20
        assert lib.rfx_plan_add_time_cond(plan, ctypes.byref(tc)) == _lib.RFX_OK
        tc.min_period = 0.0
        assert lib.rfx_plan_add_time_cond(plan, ctypes.byref(tc)) == _lib.RFX_E_INVAL

        md = _lib.ModulationDesc()
        md.mode, md.n_rows, md.n_norms, md.width = _lib.RFX_ADARMS_GATE, 10, 37, 1024
        md.w = md.b = md.cond = md.a2 = md.gate = 1 << 20
        assert lib.rfx_plan_add_modulation(plan, ctypes.byref(md)) == _lib.RFX_OK
        md.mode = 7
        assert lib.rfx_plan_add_modulation(plan, ctypes.byref(md)) == _lib.RFX_E_INVAL

        q = _lib.KvQuantDesc()
        q.mode, q.in_dtype = _lib.RFX_QUANT_I8_SYM, _lib.RFX_DTYPE_BF16
        q.k = q.v = q.k_q = q.v_q = q.k_scale = q.v_scale = 1 << 20
        q.B, q.H, q.L, q.D, q.capacity = 1, 1, 768, 256, 2048
        q.xs_b, q.xs_h, q.xs_l = 768 * 256, 768 * 256, 256
        q.qs_b, q.qs_h, q.qs_c = 2048 * 256, 2048 * 256, 256
        q.ss_b, q.ss_h, q.ss_c = 2048, 2048, 1
        q.region_base, q.region_off, q.region_len = 0, 1280, 2048
        assert lib.rfx_plan_add_kv_quant(plan, ctypes.byref(q)) == _lib.RFX_OK
        q.region_len = 4096  # the region runs past the ring's capacity
        assert lib.rfx_plan_add_kv_quant(plan, ctypes.byref(q)) == _lib.RFX_E_INVAL

        ln = _lib.LayerNormDesc()
        ln.T, ln.C = 768, 1004  # C % 8 != 0
        ln.x = ln.y = ln.w = ln.b = 1 << 20
        ln.ldx = ln.ldy = 1024
        assert lib.rfx_plan_add_layer_norm(plan, ctypes.byref(ln)) == _lib.RFX_E_INVAL
        va = _lib.VitAttnDesc()
        va.B, va.N, va.H, va.D = 3, 300, 16, 72  # more than 256 tokens per image
        va.qkv = va.out = 1 << 20
        va.ld_qkv, va.ld_out, va.scale = 3 * 16 * 72, 16 * 72, 72 ** -0.5
        assert lib.rfx_plan_add_vit_attention(plan, ctypes.byref(va)) == _lib.RFX_E_INVAL
        pd = _lib.PatchesDesc()
        pd.B, pd.C, pd.H, pd.W, pd.patch = 3, 3, 224, 220, 14  # not square
        pd.image = pd.out = 1 << 20
        pd.ldo = 640
        assert lib.rfx_plan_add_patches(plan, ctypes.byref(pd)) == _lib.RFX_E_INVAL

        assert lib.rfx_plan_num_launches(plan, ctypes.byref(n)) == _lib.RFX_OK
        assert n.value == 1 + 1 + 3 + 1 + 1
        # empty ops are accepted and launch nothing
        q.region_len, q.L = 2048, 0
        assert lib.rfx_plan_add_kv_quant(plan, ctypes.byref(q)) == _lib.RFX_OK
        assert lib.rfx_kv_quant_append(ctypes.byref(q), None) == _lib.RFX_OK
        cp.dst_row_offset, cp.rows = 1, 0
        assert lib.rfx_plan_add_copy_rows(plan, ctypes.byref(cp)) == _lib.RFX_OK
        assert lib.rfx_copy_rows(ctypes.byref(cp), None) == _lib.RFX_OK
        assert lib.rfx_plan_num_launches(plan, ctypes.byref(n)) == _lib.RFX_OK
        assert n.value == 1 + 1 + 3 + 1 + 1
    finally:
        assert lib.rfx_plan_destroy(plan) == _lib.RFX_OK


@pytest.mark.parametrize("T,O,K,want", [
    (768, 2048, 16384, 65536 + 96 * 3 * 128 * 128 * 4),  # down_proj of a 768-token frame: 96 tiles, K split 3
    (768, 32768, 2048, 0),                              # gate/up: 768 tiles fill the SMs
    (50, 2048, 16384, 0),                               # few tokens: the per-tile kernel
])
def test_linear_split_workspace_size(T, O, K, want):
    """The split-K workspace query needs no device: a fixed 64 KB counter block
    plus fp32 partial slots [tile][split][128 tokens][128 rows] (148 SMs
    assumed when no GPU answers)."""
    lib = _lib.load()
    d = _lib.LinearDesc()
    d.T, d.O, d.K, d.tokens_per_batch = T, O, K, T
    d.prologue, d.epilogue = _lib.RFX_PRO_LOAD, _lib.RFX_EPI_STORE
    d.w, d.x, d.y = 1 << 20, 2 << 20, 3 << 20
    d.ldx, d.ldy = K, O
    n = ctypes.c_size_t(7)
    assert lib.rfx_linear_workspace_size(ctypes.byref(d), ctypes.byref(n)) == _lib.RFX_OK
    assert n.value == want


def test_kv_quant_rejects_too_many_rings():
    """B * H above 65535 (one grid row per (b, h)) is refused before any launch."""
    lib = _lib.load()
    d = _lib.KvQuantDesc()
    d.mode, d.in_dtype = _lib.RFX_QUANT_I8_SYM, _lib.RFX_DTYPE_BF16
    d.k = d.v = d.k_q = d.v_q = d.k_scale = d.v_scale = 1 << 20  # aligned, never dereferenced
    d.B, d.H, d.L, d.D, d.capacity = 65536, 1, 1, 256, 1
    d.xs_b = d.xs_h = d.xs_l = 256
    d.qs_b = d.qs_h = d.qs_c = 256
    d.ss_b = d.ss_h = d.ss_c = 1
    d.region_base, d.region_off, d.region_len = 0, 0, 1
    assert lib.rfx_kv_quant_append(ctypes.byref(d), None) == _lib.RFX_E_INVAL
    assert b"65535" in lib.rfx_last_error()


def test_vision_entry_points_reject_bad_shapes():
    """Shape checks of the vision tower's entry points run before any launch."""
    lib = _lib.load()
    a = _lib.VitAttnDesc()
    a.B, a.N, a.H, a.D = 1, 257, 16, 72  # more than 256 tokens per image
    a.qkv = a.out = 1 << 20
    a.ld_qkv, a.ld_out, a.scale = 3 * 16 * 72, 16 * 72, 0.1
    assert lib.rfx_vit_attention(ctypes.byref(a), None) == _lib.RFX_E_INVAL
    a.N, a.D = 256, 76  # head dim not a multiple of 8
    assert lib.rfx_vit_attention(ctypes.byref(a), None) == _lib.RFX_E_INVAL
    n = _lib.LayerNormDesc()
    n.T, n.C = 4, 1004  # C % 8 != 0
    n.x = n.y = n.w = n.b = 1 << 20
    n.ldx = n.ldy = 1024
    assert lib.rfx_layer_norm(ctypes.byref(n), None) == _lib.RFX_E_INVAL
    p = _lib.PatchesDesc()
    p.B, p.C, p.H, p.W, p.patch = 1, 3, 224, 224, 14
    p.image = p.out = 1 << 20
    p.ldo = 588  # not a multiple of 64
    assert lib.rfx_patches(ctypes.byref(p), None) == _lib.RFX_E_INVAL


def test_diagnostic_switches():
    """The phase stamps are left out of the default build, so asking for a
    trace buffer is refused (RFX_E_UNSUPPORTED) rather than silently ignored;
    turning tracing off and toggling the executor's cooperative launch need
    no device."""
    lib = _lib.load()
    assert lib.rfx_set_trace(None, 0) == _lib.RFX_OK
    assert lib.rfx_set_trace(1 << 20, 4096) == _lib.RFX_E_UNSUPPORTED
    assert b"RFX_TRACE" in lib.rfx_last_error()
    assert lib.rfx_set_trace(None, 0) == _lib.RFX_OK
    assert lib.rfx_set_chunk_cooperative(0) == _lib.RFX_OK
    assert lib.rfx_set_chunk_cooperative(1) == _lib.RFX_OK
