// Internal declarations shared by the CUDA translation units of librfx_b200.
#pragma once
#include <cuda_runtime.h>
#include <cuda.h>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/rfx.h"
#include "ptx.cuh"

namespace rfx {

// ---------------------------------------------------------------- errors ---
// Records a thread-local error message for rfx_last_error() and returns code.
int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
// Device address of the library's status word on the current device.
int* device_status_ptr();

// Device buffer for per-CTA phase timestamps (rfx_set_trace), or nullptr when
// tracing is off or the buffer holds fewer than n_events 8-byte slots.
void* trace_buffer(size_t n_events);

// Whether kernels are launched with programmatic dependent launch.
bool pdl_enabled();
bool chunk_cooperative();

// Bound (ns) of device waits on work of other CTAs (rfx_set_wait_limit_ns).
unsigned long long dependency_wait_limit_ns();

// ------------------------------------------------------------------ enums ---
enum QuantMode : int { kQuantI8Sym = RFX_QUANT_I8_SYM, kQuantU8Ref = RFX_QUANT_U8_REF };
enum Dtype : int { kDtypeF32 = RFX_DTYPE_F32, kDtypeBF16 = RFX_DTYPE_BF16 };

// ------------------------------------------------------------ launching ---
// cudaLaunchKernelEx with optional PDL and cluster dimensions.
int launch_kernel_impl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                       dim3 cluster, void** args);

template <typename... Args>
int launch_kernel(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, int cluster_x,
                  Args&... args) {
  void* argv[] = {static_cast<void*>(&args)...};
  return launch_kernel_impl(func, grid, block, smem, stream, pdl, dim3(cluster_x, 1, 1), argv);
}
template <typename... Args>
int launch_kernel_cluster(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                          dim3 cluster, Args&... args) {
  void* argv[] = {static_cast<void*>(&args)...};
  return launch_kernel_impl(func, grid, block, smem, stream, pdl, cluster, argv);
}

// Whether a cluster of cluster_x CTAs of this kernel can be resident at once.
bool cluster_fits(const void* func, dim3 grid, int threads, int smem, int cluster_x);

// Raises the dynamic shared-memory limit of a kernel once per process.
int ensure_smem_attr(const void* func, int bytes, bool nonportable_cluster = false);

// ----------------------------------------------------------- tensor maps ---
// 2-D row-major tensor [rows][cols] with the given element size; box
// {box_cols, box_rows}; swizzle 128B when swizzle128 is set.
int make_tmap_2d(CUtensorMap* out, const void* base, int elem_bytes, uint64_t cols, uint64_t rows,
                 uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows, bool swizzle128);

// ------------------------------------------------------- kernel launchers ---
struct KvQuantDesc {
  int mode, in_dtype;
  const void* x[2];
  long xs_b, xs_h, xs_l;
  int B, H, L, D;
  void* q[2];
  long qs_b, qs_h, qs_c;
  int capacity;
  void* scale[2];
  void* zp[2];
  long ss_b, ss_h, ss_c;
  int region_base, region_off, region_len;
};
KvQuantDesc kv_quant_internal(const rfx_kv_quant_desc& d);
int launch_kv_quant_append(const KvQuantDesc& d, cudaStream_t stream, bool pdl);

int launch_linear(const rfx_linear_desc& d, const CUtensorMap* tmW, const CUtensorMap* tmX, cudaStream_t stream,
                  bool pdl);
int build_linear_maps(const rfx_linear_desc& d, CUtensorMap* tmW, CUtensorMap* tmX);

int launch_attention(const rfx_attn_desc& d, const CUtensorMap* tmQ, const CUtensorMap* tmK, const CUtensorMap* tmV,
                     cudaStream_t stream, bool pdl);
int build_attention_maps(const rfx_attn_desc& d, CUtensorMap* tmQ, CUtensorMap* tmK, CUtensorMap* tmV);
size_t attention_workspace_bytes(const rfx_attn_desc& d);
// Kernel launches of one rfx_attention call: the dense conversion (dense
// source), the attention, and the split-KV combine (more than one split).
int attention_launches(const rfx_attn_desc& d);

// Descriptor checks of the launchers below, host-only (no CUDA call): each
// launcher runs its check first, and the plan adds run it when an op is added.
int validate_kv_quant(const KvQuantDesc& d);
int validate_time_cond(const rfx_time_cond_desc& d);
int validate_modulation(const rfx_modulation_desc& d);
int validate_io(const rfx_action_io_desc& d, bool tail);
int validate_copy_rows(const rfx_copy_rows_desc& d);
int validate_rms_norm(const rfx_norm_desc& d);
int validate_patches(const rfx_patches_desc& d);
int validate_layer_norm(const rfx_layer_norm_desc& d);
int validate_vit_attention(const rfx_vit_attn_desc& d);

int launch_time_cond(const rfx_time_cond_desc& d, cudaStream_t stream, bool pdl);
int launch_modulation(const rfx_modulation_desc& d, cudaStream_t stream, bool pdl);
int launch_action_in(const rfx_action_io_desc& d, cudaStream_t stream, bool pdl);
int launch_euler_tail(const rfx_action_io_desc& d, cudaStream_t stream, bool pdl);
int launch_copy_rows(const rfx_copy_rows_desc& d, cudaStream_t stream, bool pdl);
int launch_rms_norm(const rfx_norm_desc& d, cudaStream_t stream, bool pdl);
int launch_patches(const rfx_patches_desc& d, cudaStream_t stream, bool pdl);
int launch_layer_norm(const rfx_layer_norm_desc& d, cudaStream_t stream, bool pdl);
int launch_vit_attention(const rfx_vit_attn_desc& d, cudaStream_t stream, bool pdl);
int run_chunk_op(rfx_chunk* c, cudaStream_t s);

}  // namespace rfx
