// Runtime of librfx_b200: error reporting, launch helper (programmatic
// dependent launch + clusters), TMA descriptor encoding, the device status
// word, and execution plans (ordered launch lists with CUDA-graph capture).
#include "rfx_internal.h"

#include <atomic>
#include <cstdarg>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <variant>
#include <vector>

namespace rfx {

// ------------------------------------------------------------------ errors ---
namespace {
thread_local char g_last_error[512] = "";
std::atomic<bool> g_pdl{true};
std::atomic<bool> g_chunk_coop{true};
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return RFX_OK;
  return set_error(RFX_E_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed); }
bool chunk_cooperative() { return g_chunk_coop.load(std::memory_order_relaxed); }

namespace {
std::atomic<unsigned long long> g_dep_wait_ns{kWaitLimitNs};
}  // namespace
unsigned long long dependency_wait_limit_ns() { return g_dep_wait_ns.load(std::memory_order_relaxed); }

// ------------------------------------------------------------ tracing ---
namespace {
std::atomic<void*> g_trace_buf{nullptr};
std::atomic<size_t> g_trace_bytes{0};
}  // namespace

void* trace_buffer(size_t n_events) {
  void* b = g_trace_buf.load();
  return (b && n_events * 8 <= g_trace_bytes.load()) ? b : nullptr;
}

// ------------------------------------------------------------ status word ---
namespace {
__device__ int g_device_status = 0;
std::mutex g_status_mu;
std::unordered_map<int, int*> g_status_ptrs;
}  // namespace

int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  auto it = g_status_ptrs.find(dev);
  if (it != g_status_ptrs.end()) return it->second;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
  g_status_ptrs[dev] = static_cast<int*>(p);
  return static_cast<int*>(p);
}

// ------------------------------------------------------------- launching ---
int launch_kernel_impl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                       dim3 cluster, void** args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  unsigned n = 0;
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster.x * cluster.y * cluster.z > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = cluster.x;
    attrs[n].val.clusterDim.y = cluster.y;
    attrs[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return check_cuda(cudaLaunchKernelExC(&cfg, func, args), "kernel launch");
}

int ensure_smem_attr(const void* func, int bytes, bool nonportable_cluster) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> done;  // per process; attributes are per device but identical
  std::lock_guard<std::mutex> lk(mu);
  int dev = 0;
  cudaGetDevice(&dev);
  const void* key = reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(func) ^ (static_cast<uintptr_t>(dev) << 48));
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return RFX_OK;
  int rc = check_cuda(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                      "cudaFuncSetAttribute(smem)");
  if (rc) return rc;
  // one carveout (all shared memory) for every kernel of the library, so the
  // SMs are not re-partitioned between consecutive launches
  rc = check_cuda(cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, 100),
                  "cudaFuncSetAttribute(carveout)");
  if (rc) return rc;
  if (nonportable_cluster) {
    rc = check_cuda(cudaFuncSetAttribute(func, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                    "cudaFuncSetAttribute(non-portable cluster)");
    if (rc) return rc;
  }
  done[key] = bytes;
  return RFX_OK;
}

bool cluster_fits(const void* func, dim3 grid, int threads, int smem, int cluster_x) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, bool> memo;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t key = (reinterpret_cast<uintptr_t>(func) * 1315423911ull) ^ (static_cast<uint64_t>(smem) << 20) ^
                       (static_cast<uint64_t>(cluster_x) << 8) ^ static_cast<uint64_t>(dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = cluster_x;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  const bool ok = cudaOccupancyMaxActiveClusters(&n, func, &cfg) == cudaSuccess && n > 0;
  cudaGetLastError();
  std::lock_guard<std::mutex> lk(mu);
  memo[key] = ok;
  return ok;
}

// ------------------------------------------------------------ tensor maps ---
namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

int make_tmap_2d(CUtensorMap* out, const void* base, int elem_bytes, uint64_t cols, uint64_t rows,
                 uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(RFX_E_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (!base || (reinterpret_cast<uintptr_t>(base) & 15u) || (row_stride_bytes & 15u) || rows == 0 || cols == 0)
    return set_error(RFX_E_INVAL, "tensor map: base/stride must be 16-byte aligned and shape non-empty");
  CUtensorMapDataType dt;
  switch (elem_bytes) {
    case 1: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
    case 2: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case 4: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    default: return set_error(RFX_E_INVAL, "tensor map: element size");
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(RFX_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return RFX_OK;
}

}  // namespace rfx

// ================================================================ C ABI ====
using namespace rfx;

extern "C" int rfx_version(void) { return 100; }

extern "C" const char* rfx_last_error(void) { return g_last_error; }

extern "C" int rfx_set_trace(void* buf, size_t bytes) {
  if (buf && (reinterpret_cast<uintptr_t>(buf) & 7u)) return set_error(RFX_E_INVAL, "rfx_set_trace: 8-byte alignment");
  if (buf && !kTraceBuilt)
    return set_error(RFX_E_UNSUPPORTED,
                     "rfx_set_trace: this library was built without the phase stamps; rebuild it with "
                     "make -C reflex_b200/csrc EXTRA_NVFLAGS=-DRFX_TRACE");
  g_trace_bytes.store(buf ? bytes : 0);
  g_trace_buf.store(buf);
  return RFX_OK;
}

extern "C" int rfx_set_wait_limit_ns(unsigned long long ns) {
  g_dep_wait_ns.store(ns == 0 ? kWaitLimitNs : ns);
  return RFX_OK;
}

extern "C" int rfx_set_chunk_cooperative(int enable) {
  g_chunk_coop.store(enable != 0);
  return RFX_OK;
}

extern "C" int rfx_set_pdl(int enable) {
  g_pdl.store(enable != 0);
  return RFX_OK;
}

extern "C" int rfx_num_sms(int* out) {
  if (!out) return set_error(RFX_E_INVAL, "rfx_num_sms: null");
  static std::mutex mu;
  static std::unordered_map<int, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(RFX_E_CUDA, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) {
    *out = it->second;
    return RFX_OK;
  }
  int n = 0;
  int rc = check_cuda(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
  if (rc) return rc;
  cache[dev] = n;
  *out = n;
  return RFX_OK;
}

extern "C" int rfx_device_status(void* stream, int* out) {
  if (!out) return set_error(RFX_E_INVAL, "rfx_device_status: null");
  int* p = device_status_ptr();
  if (!p) return set_error(RFX_E_CUDA, "rfx_device_status: no device status word");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0, zero = 0;
  int rc = check_cuda(cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, s), "status read");
  if (rc) return rc;
  rc = check_cuda(cudaMemcpyAsync(p, &zero, sizeof(int), cudaMemcpyHostToDevice, s), "status clear");
  if (rc) return rc;
  rc = check_cuda(cudaStreamSynchronize(s), "status sync");
  if (rc) return rc;
  *out = v;
  return RFX_OK;
}

namespace rfx {
KvQuantDesc kv_quant_internal(const rfx_kv_quant_desc& d) {
  KvQuantDesc k{};
  k.mode = d.mode;
  k.in_dtype = d.in_dtype;
  k.x[0] = d.k;
  k.x[1] = d.v;
  k.xs_b = d.xs_b;
  k.xs_h = d.xs_h;
  k.xs_l = d.xs_l;
  k.B = d.B;
  k.H = d.H;
  k.L = d.L;
  k.D = d.D;
  k.q[0] = d.k_q;
  k.q[1] = d.v_q;
  k.qs_b = d.qs_b;
  k.qs_h = d.qs_h;
  k.qs_c = d.qs_c;
  k.capacity = d.capacity;
  k.scale[0] = d.k_scale;
  k.scale[1] = d.v_scale;
  k.zp[0] = d.k_zp;
  k.zp[1] = d.v_zp;
  k.ss_b = d.ss_b;
  k.ss_h = d.ss_h;
  k.ss_c = d.ss_c;
  k.region_base = d.region_base;
  k.region_off = d.region_off;
  k.region_len = d.region_len;
  return k;
}
}  // namespace rfx

extern "C" int rfx_kv_quant_append(const rfx_kv_quant_desc* d, void* stream) {
  if (!d) return set_error(RFX_E_INVAL, "rfx_kv_quant_append: null descriptor");
  return launch_kv_quant_append(kv_quant_internal(*d), static_cast<cudaStream_t>(stream), pdl_enabled());
}

// ================================================================ plans ====
namespace {
struct LinearOp {
  rfx_linear_desc d;
  CUtensorMap w, x;
};
struct AttnOp {
  rfx_attn_desc d;
  CUtensorMap q, k, v;
};
struct QuantOp {
  rfx_kv_quant_desc d;
};
struct TimeOp {
  rfx_time_cond_desc d;
};
struct ModOp {
  rfx_modulation_desc d;
};
struct InOp {
  rfx_action_io_desc d;
};
struct TailOp {
  rfx_action_io_desc d;
};
struct CopyOp {
  rfx_copy_rows_desc d;
};
struct NormOp {
  rfx_norm_desc d;
};
struct PatchOp {
  rfx_patches_desc d;
};
struct LayerNormOp {
  rfx_layer_norm_desc d;
};
struct VitAttnOp {
  rfx_vit_attn_desc d;
};
struct BarrierOp {};
struct ChunkOp {
  rfx_chunk* c;
};
using Op = std::variant<LinearOp, AttnOp, QuantOp, TimeOp, ModOp, InOp, TailOp, CopyOp, NormOp, BarrierOp, ChunkOp,
                        PatchOp, LayerNormOp, VitAttnOp>;
}  // namespace

struct rfx_plan {
  std::vector<Op> ops;
  int launches = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int device = -1;
};

namespace {
int run_op(const Op& op, cudaStream_t s, bool pdl) {
  if (auto* o = std::get_if<LinearOp>(&op)) return launch_linear(o->d, &o->w, &o->x, s, pdl);
  if (auto* o = std::get_if<AttnOp>(&op)) return launch_attention(o->d, &o->q, &o->k, &o->v, s, pdl);
  if (auto* o = std::get_if<QuantOp>(&op)) return launch_kv_quant_append(kv_quant_internal(o->d), s, pdl);
  if (auto* o = std::get_if<TimeOp>(&op)) return launch_time_cond(o->d, s, pdl);
  if (auto* o = std::get_if<ModOp>(&op)) return launch_modulation(o->d, s, pdl);
  if (auto* o = std::get_if<InOp>(&op)) return launch_action_in(o->d, s, pdl);
  if (auto* o = std::get_if<TailOp>(&op)) return launch_euler_tail(o->d, s, pdl);
  if (auto* o = std::get_if<CopyOp>(&op)) return launch_copy_rows(o->d, s, pdl);
  if (auto* o = std::get_if<NormOp>(&op)) return launch_rms_norm(o->d, s, pdl);
  if (auto* o = std::get_if<ChunkOp>(&op)) return run_chunk_op(o->c, s);
  if (auto* o = std::get_if<PatchOp>(&op)) return launch_patches(o->d, s, pdl);
  if (auto* o = std::get_if<LayerNormOp>(&op)) return launch_layer_norm(o->d, s, pdl);
  if (auto* o = std::get_if<VitAttnOp>(&op)) return launch_vit_attention(o->d, s, pdl);
  return set_error(RFX_E_STATE, "plan: unknown op");
}
// Launches every op in order; an op that follows a BarrierOp runs without PDL.
int run_ops(const std::vector<Op>& ops, cudaStream_t s, bool pdl) {
  bool serialize = false;
  for (const Op& op : ops) {
    if (std::holds_alternative<BarrierOp>(op)) {
      serialize = true;
      continue;
    }
    int rc = run_op(op, s, pdl && !serialize);
    if (rc) return rc;
    serialize = false;
  }
  return RFX_OK;
}
void release_graph(rfx_plan* p) {
  if (p->exec) cudaGraphExecDestroy(p->exec);
  if (p->graph) cudaGraphDestroy(p->graph);
  p->exec = nullptr;
  p->graph = nullptr;
}
}  // namespace

extern "C" int rfx_plan_create(rfx_plan** out) {
  if (!out) return set_error(RFX_E_INVAL, "rfx_plan_create: null");
  *out = new (std::nothrow) rfx_plan();
  if (!*out) return set_error(RFX_E_INVAL, "rfx_plan_create: out of host memory");
  cudaGetDevice(&(*out)->device);
  return RFX_OK;
}

extern "C" int rfx_plan_destroy(rfx_plan* plan) {
  if (!plan) return RFX_OK;
  release_graph(plan);
  delete plan;
  return RFX_OK;
}

#define PLAN_GUARD(plan)                                                       \
  do {                                                                         \
    if (!(plan) || !desc) return set_error(RFX_E_INVAL, "plan: null argument"); \
    if ((plan)->exec) return set_error(RFX_E_STATE, "plan: already captured"); \
  } while (0)

extern "C" int rfx_plan_add_linear(rfx_plan* plan, const rfx_linear_desc* desc) {
  PLAN_GUARD(plan);
  LinearOp op{*desc, {}, {}};
  int rc = build_linear_maps(op.d, &op.w, &op.x);
  if (rc) return rc;
  plan->ops.emplace_back(op);
  plan->launches += 1;
  return RFX_OK;
}
extern "C" int rfx_plan_add_attention(rfx_plan* plan, const rfx_attn_desc* desc) {
  PLAN_GUARD(plan);
  AttnOp op{*desc, {}, {}, {}};
  int rc = build_attention_maps(op.d, &op.q, &op.k, &op.v);
  if (rc) return rc;
  const size_t ws = attention_workspace_bytes(op.d);
  if (ws > 0 && (!desc->workspace || desc->workspace_bytes < ws))
    return set_error(RFX_E_INVAL, "plan: attention needs %zu bytes of workspace", ws);
  plan->ops.emplace_back(op);
  plan->launches += attention_launches(op.d);
  return RFX_OK;
}
extern "C" int rfx_plan_add_kv_quant(rfx_plan* plan, const rfx_kv_quant_desc* desc) {
  PLAN_GUARD(plan);
  const int rc = validate_kv_quant(kv_quant_internal(*desc));
  if (rc) return rc;
  plan->ops.emplace_back(QuantOp{*desc});
  plan->launches += desc->L > 0 ? 1 : 0;  // an empty append launches nothing
  return RFX_OK;
}
extern "C" int rfx_plan_add_time_cond(rfx_plan* plan, const rfx_time_cond_desc* desc) {
  PLAN_GUARD(plan);
  const int rc = validate_time_cond(*desc);
  if (rc) return rc;
  plan->ops.emplace_back(TimeOp{*desc});
  plan->launches += desc->w_in ? 3 : 1;
  return RFX_OK;
}
extern "C" int rfx_plan_add_modulation(rfx_plan* plan, const rfx_modulation_desc* desc) {
  PLAN_GUARD(plan);
  const int rc = validate_modulation(*desc);
  if (rc) return rc;
  plan->ops.emplace_back(ModOp{*desc});
  plan->launches += 1;
  return RFX_OK;
}
extern "C" int rfx_plan_add_action_in(rfx_plan* plan, const rfx_action_io_desc* desc) {
  PLAN_GUARD(plan);
  const int rc = validate_io(*desc, false);
  if (rc) return rc;
  plan->ops.emplace_back(InOp{*desc});
  plan->launches += 1;
  return RFX_OK;
}
extern "C" int rfx_plan_add_euler_tail(rfx_plan* plan, const rfx_action_io_desc* desc) {
  PLAN_GUARD(plan);
  const int rc = validate_io(*desc, true);
  if (rc) return rc;
  plan->ops.emplace_back(TailOp{*desc});
  plan->launches += 1;
  return RFX_OK;
}

extern "C" int rfx_plan_add_copy_rows(rfx_plan* plan, const rfx_copy_rows_desc* desc) {
  PLAN_GUARD(plan);
  const int rc = validate_copy_rows(*desc);
  if (rc) return rc;
  plan->ops.emplace_back(CopyOp{*desc});
  plan->launches += desc->rows > 0 ? 1 : 0;  // no rows: nothing is launched
  return RFX_OK;
}

extern "C" int rfx_plan_add_rms_norm(rfx_plan* plan, const rfx_norm_desc* desc) {
  PLAN_GUARD(plan);
  const int rc = validate_rms_norm(*desc);
  if (rc) return rc;
  plan->ops.emplace_back(NormOp{*desc});
  plan->launches += 1;
  return RFX_OK;
}

extern "C" int rfx_plan_add_patches(rfx_plan* plan, const rfx_patches_desc* desc) {
  PLAN_GUARD(plan);
  const int rc = validate_patches(*desc);
  if (rc) return rc;
  plan->ops.emplace_back(PatchOp{*desc});
  plan->launches += 1;
  return RFX_OK;
}
extern "C" int rfx_plan_add_layer_norm(rfx_plan* plan, const rfx_layer_norm_desc* desc) {
  PLAN_GUARD(plan);
  const int rc = validate_layer_norm(*desc);
  if (rc) return rc;
  plan->ops.emplace_back(LayerNormOp{*desc});
  plan->launches += 1;
  return RFX_OK;
}
extern "C" int rfx_plan_add_vit_attention(rfx_plan* plan, const rfx_vit_attn_desc* desc) {
  PLAN_GUARD(plan);
  const int rc = validate_vit_attention(*desc);
  if (rc) return rc;
  plan->ops.emplace_back(VitAttnOp{*desc});
  plan->launches += 1;
  return RFX_OK;
}

extern "C" int rfx_plan_add_chunk(rfx_plan* plan, rfx_chunk* chunk) {
  if (!plan || !chunk) return set_error(RFX_E_INVAL, "plan: null argument");
  if (plan->exec) return set_error(RFX_E_STATE, "plan: already captured");
  plan->ops.emplace_back(ChunkOp{chunk});
  plan->launches += 1;
  return RFX_OK;
}

extern "C" int rfx_plan_add_barrier(rfx_plan* plan) {
  if (!plan) return set_error(RFX_E_INVAL, "plan: null argument");
  if (plan->exec) return set_error(RFX_E_STATE, "plan: already captured");
  plan->ops.emplace_back(BarrierOp{});
  return RFX_OK;
}

extern "C" int rfx_plan_num_launches(const rfx_plan* plan, int* out) {
  if (!plan || !out) return set_error(RFX_E_INVAL, "rfx_plan_num_launches: null");
  *out = plan->launches;
  return RFX_OK;
}

extern "C" int rfx_plan_run(rfx_plan* plan, void* stream) {
  if (!plan) return set_error(RFX_E_INVAL, "rfx_plan_run: null plan");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return run_ops(plan->ops, s, pdl_enabled());
}

extern "C" int rfx_plan_capture(rfx_plan* plan, void* stream) {
  if (!plan) return set_error(RFX_E_INVAL, "rfx_plan_capture: null plan");
  if (!stream) return set_error(RFX_E_INVAL, "rfx_plan_capture: capture needs a non-default stream");
  release_graph(plan);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = check_cuda(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  if (rc) return rc;
  const int run_rc = run_ops(plan->ops, s, pdl_enabled());
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(s, &g);
  if (run_rc) {
    if (g) cudaGraphDestroy(g);
    return run_rc;
  }
  rc = check_cuda(e, "cudaStreamEndCapture");
  if (rc) return rc;
  plan->graph = g;
  rc = check_cuda(cudaGraphInstantiate(&plan->exec, g, 0), "cudaGraphInstantiate");
  if (rc) {
    release_graph(plan);
    return rc;
  }
  return RFX_OK;
}

extern "C" int rfx_plan_replay(rfx_plan* plan, void* stream) {
  if (!plan) return set_error(RFX_E_INVAL, "rfx_plan_replay: null plan");
  if (!plan->exec) return set_error(RFX_E_STATE, "rfx_plan_replay: plan was not captured");
  return check_cuda(cudaGraphLaunch(plan->exec, static_cast<cudaStream_t>(stream)), "cudaGraphLaunch");
}
