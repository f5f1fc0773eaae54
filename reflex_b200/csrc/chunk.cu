// Persistent executor of one whole PI0.5 action chunk: all Euler steps, all
// layers and the Euler tails run inside ONE kernel launch with one CTA per SM.
//
// Why: at one robot stream the chunk is a chain of ~1,450 small dependent
// operations.  As separate launches each pays launch + setup + teardown
// (3-4 us) on top of its useful time; here each dependency costs one release
// / acquire of a global counter instead, and every CTA keeps streaming the
// weights of its next GEMM tile while the rest of the GPU works on the
// current phase.
//
// Work decomposition (T = B*S <= 64 tokens; per layer, in phase order):
//   QKV   20 row tiles x 2 K-splits on the two CTAs of a cluster: tcgen05
//         GEMM of the packed [Wq;Wk;Wv] against the normed input; each CTA
//         pushes the peer's rows of its fp32 partial through DSMEM, sums the
//         rows it finishes and applies RoPE (rows r / r+64 of a tile are the
//         rotary pair) -> q (head-major), k_new, v_new (bf16).
//   ATTN  (stream, 128-row query tile, key-block split): the partitioned
//         attention of the new tokens over the int8 context ring + the new
//         keys, on tcgen05 with TMEM accumulators (context rows are loaded and
//         converted int8 -> bf16 K / f16 V in shared memory; per-token scales
//         folded into the scores / probabilities) -> fp32 partial (O, m, l).
//   COMB  rows of a query tile: log-sum-exp merge of the partials -> bf16.
//   O     8 row tiles x 8 K-splits -> fp32 partials.
//   FIN_O per token: h += gate * bf16(sum of O partials); post-attention
//         (Ada)RMSNorm -> GEMM input.
//   GU    64 row tiles x 2 K-splits on a cluster, as QKV: GELU-tanh(gate) * up.
//   DOWN  8 row tiles x 8 K-splits -> fp32 partials.
//   FIN_D per token: h += gate * bf16(sum of down partials); next layer's
//         input norm, or after the last layer the Euler tail (final norm,
//         action_out_proj, x += dt*v, next step's action_in_proj, norm).
//
// Every phase counts its finished items on a global counter (release); the
// consumers of the phase wait for the count of the current use (acquire).
// Counters only grow within a chunk and are cleared before each chunk.
// Partials are summed in a fixed order, so results do not depend on timing.
//
// Roles (320 threads): warp 0 lane 0 streams weight / activation tiles
// through an 8-stage TMA ring (weights are issued before the tile's input is
// ready), warp 1 lane 0 issues tcgen05.mma, warps 2-9 (two per TMEM lane
// quadrant) do everything else.  The attention tiles reuse the ring's shared memory;
// the producer drains the ring before an attention item and resumes after it.
//
// Every wait is bounded (about one second); a wait that runs out records a
// device status code and raises a chunk-wide abort flag, after which every
// role leaves its loop, in-flight copies are drained and TMEM is freed.
#include "rfx_internal.h"

#include <algorithm>
#include <vector>

namespace rfx {
namespace {

constexpr int kWorkers = 256;  // worker threads: warps 2..9, two per TMEM lane quadrant
constexpr int kThreads = 64 + kWorkers;
constexpr int kNT = 64;  // token tile: T <= 64
constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kStages = 8;
constexpr int kWBytes = kBM * kBK * 2;  // 16 KB weight tile
constexpr int kXBytes = kNT * kBK * 2;  // 8 KB activation tile
constexpr int kOffX = kStages * kWBytes;
constexpr int kOffRed = kOffX + kStages * kXBytes;  // 192 KB: accumulator tile [t][128] fp32
constexpr int kRedBytes = kNT * kBM * 4;
constexpr int kOffSmall = kOffRed + kRedBytes;      // 224 KB
constexpr int kSmallBytes = 1024;
constexpr int kSmemBytes = kOffSmall + kSmallBytes + 1024;

// attention overlay on the ring region
constexpr int kD = 256, kKB = 64, kQR = 128;
constexpr int kOffAQ = 0;        // 4 x [128 x 64] bf16
constexpr int kOffAK = 65536;    // 4 x [64 x 64] bf16
constexpr int kOffAV = 98304;    // 4 x [64 x 64] f16, MN-major blocks
constexpr int kOffAP = 131072;   // [128 x 64] f16
constexpr int kOffAScales = 147456;  // 8 x 64 floats (2 KB): per-key scales, zero points, block ids (first set)
constexpr int kOffAXchg = 149504;    // 768 floats: row maxima and sums of the two column halves
constexpr int kOffAStg = 155648;     // int8 rows of one context block, K [64][256] then V [64][256]
constexpr int kStgBytes = kKB * kD;  // 16 KB per tensor
constexpr int kOffAScales1 = kOffAStg + 2 * kStgBytes;  // the second set of per-key values
// the attention tiles overlay the ring (idle while an attention item runs)
static_assert(kOffAXchg + 3072 <= kOffAStg && kOffAScales1 + 2048 <= kOffRed,
              "attention tiles must fit in the ring");

// small region (byte offsets)
constexpr int kSmFull = 0;         // 8 mbarriers
constexpr int kSmEmpty = 64;       // 8 mbarriers
constexpr int kSmAccFull = 128;
constexpr int kSmAccFree = 136;
constexpr int kSmQFull = 144;
constexpr int kSmConv = 152;
constexpr int kSmSFull = 160;
constexpr int kSmPReady = 168;
constexpr int kSmOFull = 176;
constexpr int kSmAttnDone = 184;
constexpr int kSmTmem = 192;
constexpr int kSmKvnFull = 200;    // mbarrier: the new keys' K / V tiles (TMA) have landed
constexpr int kSmPairReady = 208;  // mbarrier: the peer CTA has pushed its partial into this CTA's tile buffer
constexpr int kSmPairDone = 216;   // mbarrier: the peer CTA has read its tile buffer (this CTA may push again)
constexpr int kSmMmaDrain = 224;   // mbarrier: every MMA this CTA issued has completed (teardown)
constexpr int kSmStgFull = 232;    // mbarrier: a context block's int8 rows have landed in the staging buffer
constexpr int kSmStgEmpty = 240;   // mbarrier: the workers have converted the staged block out of it
constexpr int kSmVReady = 248;     // mbarrier: the block's V tile is in sV (P.V may run)
constexpr int kSmRed8 = 320;       // 8 floats
constexpr int kSmXs = 512;         // 64 floats
static_assert(kSmXs + 256 <= kSmallBytes, "small region");

// kTAtIn / kTAtOut and kTFinAt1 / kTFinAt2: PI0's action-time MLP at the start
// of every step (modeling_pi0.py:163-200), as GEMM phases with per-token
// reductions.
enum TaskType : int { kTInit = 0, kTQkv = 1, kTO = 2, kTGu = 3, kTDown = 4, kTAttn = 5, kTComb = 6, kTFinO = 7, kTFinD = 8,
                      kTAtIn = 9, kTAtOut = 10, kTFinAt1 = 11, kTFinAt2 = 12 };
enum Op : int { kOpQkv = 0, kOpO = 1, kOpGu = 2, kOpDown = 3, kOpAtIn = 4, kOpAtOut = 5, kNumOps = 6 };
enum Variant : int { kPi05 = 0, kPi0 = 1 };
// GEMM op of a task type, or -1
__host__ __device__ constexpr int gemm_op(int ty) {
  return (ty >= kTQkv && ty <= kTDown) ? ty - kTQkv : ty == kTAtIn ? kOpAtIn : ty == kTAtOut ? kOpAtOut : -1;
}
// counter lines (32 u32 = 128 B apart)
enum CtrLine : int { kCXn = 0, kCQkv = 1, kCAttn = 2, kCComb = 3, kCPo = 4, kCXn2 = 5, kCAct = 6, kCPd = 7, kCAbort = 8,
                     kCAtX = 9, kCPat1 = 10, kCAtH = 11, kCPat2 = 12, kNumCtrLines = 16 };


enum ChunkError : int { kDevTimeoutDependency = 8 };

struct OpCfg {
  int rows;    // weight rows per layer
  int K;       // reduction length
  int m_tiles;
  int splits;
  int kb;      // k-blocks per split
  float* part; // [m_tiles][splits][kNT][128] fp32
};

struct ChunkParams {
  int T, S, B, NL, steps, W, Hq, F, A, NN;
  int variant;  // kPi05 / kPi0
  int SA, TA;   // action tokens per stream / in all (PI0: S = SA + 1, the state token first)
  int n_ctx, cap, mode, scale_bf16;
  int q_tiles, attn_splits, n_ctx_blocks, n_blocks;
  int n_attn, n_comb, n_fin;
  float eps, dt, scale_log2;
  OpCfg op[kNumOps];
  const float* a1;    // [NN][W]
  const float* a2;    // [steps][NN][W] or null
  const float* b2;
  const float* gate;
  const __nv_bfloat16* w_in;   // [W][A]
  const __nv_bfloat16* b_in;   // [W]
  const __nv_bfloat16* w_out;  // [A][W]
  const __nv_bfloat16* b_out;  // [A]
  const float* rope;
  int rope_max_pos;
  const int* pos;              // [T]
  const uint8_t* const* k_ring;  // [NL] -> [B][cap][256]
  const uint8_t* const* v_ring;
  const void* const* k_scale;    // [NL] -> [B][cap]
  const void* const* v_scale;
  const void* const* k_zp;
  const void* const* v_zp;
  const unsigned char* ctx_valid;  // [B][cap] or null
  float* x;                    // [B][S][A]
  __nv_bfloat16* h;            // [T][W]
  __nv_bfloat16* xn;           // [T][W]
  __nv_bfloat16* q;            // [B][Hq][S][256], f16 bits (values rounded to bf16 first)
  __nv_bfloat16* kn;           // [T][256], f16 bits as q
  __nv_bfloat16* vn;           // [T][256], f16 bits as q
  __nv_bfloat16* attn_out;     // [T][Hq*256]
  __nv_bfloat16* act;          // [T][F]
  float* ws_o;
  float2* ws_ml;
  unsigned* ctr;
  const int4* step_tasks;
  const int* step_off;         // [grid + 1]
  const int4* init_tasks;
  const int* init_off;
  int* status;
  unsigned long long* trace;  // [grid][trace_tasks][16] stamps + task of the first step, or null
  int trace_tasks;
  unsigned long long dep_limit_ns;  // bound of a wait on another CTA's phase counter (rfx_set_wait_limit_ns)
  // PI0 only
  const float* state;            // [B][SD]
  int SD;
  const __nv_bfloat16* w_st;     // [W][SD] state_proj
  const __nv_bfloat16* b_st;     // [W]
  const float* b_atin;           // [W] action_time_mlp_in bias
  const float* b_atout;          // [W] action_time_mlp_out bias
  const __nv_bfloat16* temb;     // [steps][W] bf16 sinusoidal time embedding
  __nv_bfloat16* at_x;           // [TA][2W]: [action_in(x), time embedding]
  __nv_bfloat16* at_hid;         // [TA][W]
  __nv_bfloat16* st_emb;         // [B][W]
  const int* new_block;          // [S] block ids of the new tokens, or null (all see all)
  __nv_bfloat16* dbg_h;     // [NL][T][W] step-0 residual stream after each layer, or null
  __nv_bfloat16* dbg_attn;  // [NL][T][Hq*256] step-0 attention output of each layer, or null
};

struct Maps {
  CUtensorMap w[kNumOps];
  CUtensorMap x[kNumOps];
  CUtensorMap q;
  CUtensorMap kn;  // the new tokens' keys, f16 [B*S][256]
  CUtensorMap vn;  // the new tokens' values, f16 [B*S][256]
};

// ------------------------------------------------------------ sync helpers ---
__device__ __forceinline__ unsigned* ctr_ptr(const ChunkParams& p, int line) { return p.ctr + line * 32; }

__device__ __forceinline__ bool aborted(const ChunkParams& p) {
  return *reinterpret_cast<volatile unsigned*>(ctr_ptr(p, kCAbort)) != 0u;
}
__device__ __forceinline__ void raise_abort(const ChunkParams& p, int code) {
  record_error(p.status, code);
  atomicExch(ctr_ptr(p, kCAbort), 1u);
}
// Bounded mbarrier wait that also gives up when the chunk was aborted.
__device__ bool bar_wait(const ChunkParams& p, uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (aborted(p)) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_abort(p, code);
      return false;
    }
  }
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* a) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* a) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
// Bounded wait until a phase counter reaches `target`.  Polls with relaxed
// loads (an acquire load per poll would keep invalidating the SM's L1) and
// makes the success an acquire with one acquire load.
__device__ bool ctr_wait(const ChunkParams& p, int line, unsigned target) {
  const unsigned* c = ctr_ptr(p, line);
  if (ld_relaxed_gpu(c) >= target) {
    ld_acquire_gpu(c);
    return true;
  }
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    // back-to-back polls: each is an L2 round trip (a sleep between them only
    // delays the hand-off: 7.93 against 7.89 ms per PI0.5 chunk)
    for (int i = 0; i < 16; ++i) {
      if (ld_relaxed_gpu(c) >= target) {
        ld_acquire_gpu(c);  // the success becomes an acquire (one load, no full fence)
        return true;
      }
    }
    if (aborted(p)) return false;
    if (globaltimer_ns() - t0 > p.dep_limit_ns) {
      raise_abort(p, kDevTimeoutDependency);
      return false;
    }
  }
}
__device__ __forceinline__ void ctr_signal(const ChunkParams& p, int line) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr_ptr(p, line)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Arrive (release, cluster scope) on an mbarrier of the peer CTA of the pair.
__device__ __forceinline__ void mbar_arrive_peer(uint64_t* local_bar, uint32_t peer) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(mapa_shared(smem_u32(local_bar), peer))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait (acquire at cluster scope) that gives up on an aborted chunk.
__device__ bool bar_wait_cluster(const ChunkParams& p, uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (aborted(p)) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_abort(p, code);
      return false;
    }
  }
}

// named barrier 1 over the 256 worker threads
__device__ __forceinline__ void workers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// named barrier 2 + quad over the two worker warps that share a TMEM lane quadrant
__device__ __forceinline__ void quad_pair_sync(int quad) { asm volatile("bar.sync %0, 64;" ::"r"(2 + quad) : "memory"); }
__device__ __forceinline__ bool workers_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}
// One worker waits for the counter (acquire); the barrier that follows orders
// every worker's later reads after it.  All workers agree on the outcome.
__device__ __forceinline__ bool workers_ctr_wait(const ChunkParams& p, int et, int line, unsigned target) {
  bool ok = true;
  if (et == 0) ok = ctr_wait(p, line, target);
  return workers_all(ok);
}
// All workers' global writes are ordered before the barrier; one worker then
// releases the phase counter (the reduction's release semantics are
// cumulative, covering the writes the barrier ordered before it).
__device__ __forceinline__ void workers_publish(const ChunkParams& p, int et, int line) {
  workers_sync();
  if (et == 0) ctr_signal(p, line);
}

__device__ __forceinline__ void stamp(unsigned long long* slot, int k) {
  if (kTraceBuilt && slot) slot[k] = globaltimer_ns();
}

// ---------------------------------------------------------------- math ---
__device__ __forceinline__ float gelu_tanh(float x) {
  const float kBeta = 0.7978845608028654f;  // sqrt(2/pi)
  const float kKappa = 0.044715f;
  const float inner = kBeta * (x + kKappa * x * x * x);
  return 0.5f * x * (1.f + tanhf(inner));
}
__device__ __forceinline__ void unpack4_bf16(uint2 raw, float (&f)[4]) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}
__device__ __forceinline__ uint2 pack4_bf16(const float (&y)[4]) {
  return make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
}
__device__ __forceinline__ float load_scalar(const void* ptr, long i, bool bf16) {
  return bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(ptr)[i]) : static_cast<const float*>(ptr)[i];
}
__device__ __forceinline__ float round_to(float x, bool bf16) { return bf16 ? bf16_round(x) : x; }

// Per-op GEMM configuration; a switch keeps the parameter accesses static
// (a runtime index into the kernel parameters would copy them to local memory).
__device__ __forceinline__ OpCfg op_cfg(const ChunkParams& p, int op) {
  switch (op) {
    case kOpQkv: return p.op[kOpQkv];
    case kOpO: return p.op[kOpO];
    case kOpGu: return p.op[kOpGu];
    case kOpDown: return p.op[kOpDown];
    case kOpAtIn: return p.op[kOpAtIn];
    default: return p.op[kOpAtOut];
  }
}

// Modulation vectors of norm n at Euler step tau ([steps][NN][W]).
__device__ __forceinline__ long mod_off(const ChunkParams& p, int tau, int n) {
  return (static_cast<long>(tau) * p.NN + n) * p.W;
}

// Norm vectors of one norm for the worker's 4 features (f0 = et*4).
struct NormVec {
  float a1[4], a2[4], b2[4];
};
__device__ __forceinline__ void load4(const float* src, float (&dst)[4]) {
  *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(src);
}
__device__ __forceinline__ void load_norm_vec(const ChunkParams& p, int et, int tau, int n, NormVec& v) {
  const int f0 = et * 4;
  load4(p.a1 + static_cast<long>(n) * p.W + f0, v.a1);
  if (p.a2) load4(p.a2 + mod_off(p, tau, n) + f0, v.a2);
  if (p.b2) load4(p.b2 + mod_off(p, tau, n) + f0, v.b2);
}

// (Ada)RMSNorm of one token row held as 4 features per worker thread:
// y = ((x*rstd)*a1)*a2 + b2 (fp32, rounded by the caller), rstd =
// rsqrt(mean(x^2) + eps); the sum of squares per thread, then per warp, then
// over the eight warps in order.
__device__ void norm_row(const ChunkParams& p, int et, const float (&hv)[4], const NormVec& v, float* red8,
                         float (&y)[4]) {
  const int lane = et & 31, wq = et >> 5;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss = fmaf(hv[e], hv[e], ss);
  ss = warp_sum(ss);
  if (lane == 0) red8[wq] = ss;
  workers_sync();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kWorkers / 32; ++w) tot += red8[w];
  const float rstd = rsqrtf(tot / static_cast<float>(p.W) + p.eps);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float x = __fmul_rn(__fmul_rn(hv[e], rstd), v.a1[e]);
    if (p.a2) x = __fmul_rn(x, v.a2[e]);
    if (p.b2) x = __fadd_rn(x, v.b2[e]);
    y[e] = x;
  }
  workers_sync();  // red8 is reused by the next row
}

// h_row[o] = bf16(sum_a xs[a] * W[o][a] + b[o]) for the worker's 4 features
// (action_in_proj, or PI0's state_proj).
__device__ __forceinline__ void proj_in4(const ChunkParams& p, int et, const float* xs, float (&hv)[4],
                                         const __nv_bfloat16* w, const __nv_bfloat16* bias, int n_in) {
#pragma unroll 1
  for (int e = 0; e < 4; ++e) {
    const int o = et * 4 + e;
    const __nv_bfloat16* wr = w + static_cast<long>(o) * n_in;
    float acc = 0.f;
    for (int a = 0; a < n_in; a += 8) {
      const uint4 raw = *reinterpret_cast<const uint4*>(wr + a);
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(w2[q]);
        acc = fmaf(f.x, xs[a + 2 * q], acc);
        acc = fmaf(f.y, xs[a + 2 * q + 1], acc);
      }
    }
    hv[e] = bf16_round(acc + (bias ? __bfloat162float(bias[o]) : 0.f));
  }
}
__device__ __forceinline__ void action_in4(const ChunkParams& p, int et, const float* xs, float (&hv)[4]) {
  proj_in4(p, et, xs, hv, p.w_in, p.b_in, p.A);
}

// PI0: the action rows of the next action-time MLP input, [action_in(x), t_emb(tau)].
__device__ __forceinline__ void write_at_x(const ChunkParams& p, int et, int at, int tau, const float (&hv)[4]) {
  const int f0 = et * 4;
  __nv_bfloat16* row = p.at_x + static_cast<long>(at) * 2 * p.W;
  *reinterpret_cast<uint2*>(row + f0) = pack4_bf16(hv);
  *reinterpret_cast<uint2*>(row + p.W + f0) =
      *reinterpret_cast<const uint2*>(p.temb + static_cast<long>(tau) * p.W + f0);
}

// Sum of the split-K partials [m][split][t][128] of op for token row t, the
// worker's 4 features, in split order.
__device__ __forceinline__ void sum_partials4(const ChunkParams& p, int op, int t, int f0, float (&acc)[4]) {
  const OpCfg oc = op_cfg(p, op);
  const int m = f0 / kBM, r0 = f0 % kBM;
  acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
  for (int s0 = 0; s0 < oc.splits; s0 += 4) {
    float4 a[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (s0 + q < oc.splits) {
        const float* ps = oc.part + ((static_cast<long>(m) * oc.splits + s0 + q) * kNT + t) * kBM + r0;
        a[q] = __ldcg(reinterpret_cast<const float4*>(ps));
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (s0 + q < oc.splits) {
        acc[0] += a[q].x; acc[1] += a[q].y; acc[2] += a[q].z; acc[3] += a[q].w;
      }
    }
  }
}

// ------------------------------------------------------- worker: GEMM tile ---
// Accumulator (row = TMEM lane, 64 token columns) -> o_proj / down_proj: fp32
// partial in global memory.  QKV / gate-up: the tile's two K splits run on
// the two CTAs of a cluster, which sum them through shared memory and each
// finish half of the rows.  Returns false when the chunk was aborted.
__device__ __forceinline__ bool worker_gemm(const ChunkParams& p, uint8_t* smem, uint8_t* small, uint32_t tmem, int et, int op,
                            int layer, int m, int split, uint32_t& acc_cnt, uint32_t& pair_cnt,
                            unsigned long long* ts) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3;
  const int row = quad * 32 + lane;
  const int ch = et >> 7;  // this warp's half of the 64 token columns
  uint64_t* acc_full = reinterpret_cast<uint64_t*>(small + kSmAccFull);
  uint64_t* acc_free = reinterpret_cast<uint64_t*>(small + kSmAccFree);
  const OpCfg oc = op_cfg(p, op);
  // QKV / gate-up tiles are split along K over the two CTAs of a cluster;
  // CTA rank h runs the epilogue of row pairs (i, i+64), i in [32h, 32h+32).
  // RoPE cos / sin of this thread's epilogue items (item k: it = et + 256 k,
  // token it / 8, rows 32h + (it % 8) * 4) are fetched while the MMA runs.
  const bool paired = op == kOpQkv || op == kOpGu;
  const int half = split;
  constexpr int kItems = kNT * 8 / kWorkers;
  float4 rc[kItems], rsn[kItems];
  const bool rotary = op == kOpQkv && (m >> 1) <= p.Hq;
  if (rotary) {
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int it = et + kWorkers * k;
      if (it < p.T * 8) {
        int pos = p.pos[it >> 3];
        pos = pos < 0 ? 0 : (pos >= p.rope_max_pos ? p.rope_max_pos - 1 : pos);
        const float* cs = p.rope + static_cast<long>(pos) * 256 + (m & 1) * 64 + half * 32 + (it & 7) * 4;
        rc[k] = *reinterpret_cast<const float4*>(cs);
        rsn[k] = *reinterpret_cast<const float4*>(cs + 128);
      }
    }
  }
  bool ok = true;
  if (lane == 0) ok = bar_wait(p, acc_full, acc_cnt & 1, kDevTimeoutMmaDone);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  ++acc_cnt;
  ok = workers_all(ok);
  if (!ok) return false;
  if (et == 0) stamp(ts, 1);
  tc_fence_after();
  // accumulator rows (this thread's TMEM lane) -> o_proj / down_proj: fp32
  // partial [t][128] in global memory (summed per token by the next phase).
  // QKV / gate-up: the tile buffer [t][128] of the CTA that finishes a row
  // gathers both splits of it: the rows of quads (h, h+2) at their own
  // positions from this CTA, the peer's partial of them at row ^ 32 (rows
  // this CTA finishes nowhere else), pushed by the peer's quads (h, h+2).
  uint64_t* pair_ready = reinterpret_cast<uint64_t*>(small + kSmPairReady);
  uint64_t* pair_done = reinterpret_cast<uint64_t*>(small + kSmPairDone);
  const uint32_t peer = static_cast<uint32_t>(half ^ 1);
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* part = oc.part + (static_cast<long>(m) * oc.splits + split) * kNT * kBM;
  bool pushed = true;
  {
    // token columns 32 ch .. 32 ch + 31 of this thread's accumulator row
    uint32_t r[2][16];
#pragma unroll
    for (int c = 0; c < 2; ++c) tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + (2 * ch + c) * 16, r[c]);
    tmem_wait_ld();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(acc_free);
    if (!paired) {
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int t = (2 * ch + c) * 16 + e;
          if (t < p.T) __stcg(part + t * kBM + row, __uint_as_float(r[c][e]));
        }
    } else if ((quad & 1) == half) {
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int e = 0; e < 16; ++e) red[((2 * ch + c) * 16 + e) * kBM + row] = __uint_as_float(r[c][e]);
    } else {
      // the peer's buffer is free once the peer has read the previous tile
      if (pair_cnt > 0) {
        if (lane == 0) pushed = bar_wait_cluster(p, pair_done, (pair_cnt - 1) & 1, kDevTimeoutCluster);
        pushed = __shfl_sync(0xffffffffu, pushed ? 1 : 0, 0) != 0;
      }
      if (pushed) {
        const uint32_t dst = mapa_shared(smem_u32(red + (row ^ 32)), peer);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int t = (2 * ch + c) * 16 + e;
            if (t < p.T) st_dsmem_f32(dst + static_cast<uint32_t>(t * kBM * 4), __uint_as_float(r[c][e]));
          }
        __syncwarp();
        if (lane == 0) mbar_arrive_peer(pair_ready, peer);
      }
    }
  }
  if (et == 0) stamp(ts, 6);
  if (!paired) {
    workers_publish(p, et, op == kOpO ? kCPo : op == kOpDown ? kCPd : op == kOpAtIn ? kCPat1 : kCPat2);
    return true;
  }
  // this CTA's own rows are in its buffer (the barrier orders them for every
  // worker); then wait for the peer's pushed partial
  if (!workers_all(pushed)) return false;
  if (et == 0) stamp(ts, 8);
  {
    bool w = true;
    if (lane == 0) w = bar_wait_cluster(p, pair_ready, pair_cnt & 1, kDevTimeoutCluster);
    if (!workers_all(__shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0)) return false;
  }
  if (et == 0) stamp(ts, 9);
  // epilogue on row pairs (i, i+64), 4 rows per item: the two splits' sums
  // (two terms, so the order does not change the result)
  const int items = p.T * 8;
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int it = et + kWorkers * k;
    if (it >= items) break;
    const int t = it >> 3;
    const int i = half * 32 + (it & 7) * 4;
    const float4 va = *reinterpret_cast<const float4*>(red + t * kBM + i);
    const float4 vc = *reinterpret_cast<const float4*>(red + t * kBM + i + 64);
    const float4 pa = *reinterpret_cast<const float4*>(red + t * kBM + (i ^ 32));
    const float4 pc = *reinterpret_cast<const float4*>(red + t * kBM + ((i + 64) ^ 32));
    const float v0[4] = {va.x + pa.x, va.y + pa.y, va.z + pa.z, va.w + pa.w};
    const float v1[4] = {vc.x + pc.x, vc.y + pc.y, vc.z + pc.z, vc.w + pc.w};
    const int b = t / p.S, s = t - b * p.S;
    if (op == kOpGu) {
      float y[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float g = bf16_round(v0[j]);
        const float u = bf16_round(v1[j]);
        y[j] = __fmul_rn(bf16_round(gelu_tanh(g)), u);
      }
      *reinterpret_cast<uint2*>(p.act + static_cast<long>(t) * p.F + m * 64 + i) =
          make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
    } else {
      const int head = m >> 1;
      const int d0 = (m & 1) * 64 + i;
      float r0[4], r1[4];
      if (rotary) {
        const float cc[4] = {rc[k].x, rc[k].y, rc[k].z, rc[k].w};
        const float sn[4] = {rsn[k].x, rsn[k].y, rsn[k].z, rsn[k].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float x1 = bf16_round(v0[j]);
          const float x2 = bf16_round(v1[j]);
          r0[j] = __fsub_rn(__fmul_rn(x1, cc[j]), __fmul_rn(x2, sn[j]));
          r1[j] = __fadd_rn(__fmul_rn(x2, cc[j]), __fmul_rn(x1, sn[j]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          r0[j] = v0[j];
          r1[j] = v1[j];
        }
      }
      __nv_bfloat16* dst;
      if (head < p.Hq)
        dst = p.q + ((static_cast<long>(b) * p.Hq + head) * p.S + s) * 256;
      else if (head == p.Hq)
        dst = p.kn + static_cast<long>(t) * 256;
      else
        dst = p.vn + static_cast<long>(t) * 256;
      // q, k and v are rounded to bf16 (the reference's dtype) and kept as
      // f16 of that value (exact for |x| in [2^-14, 65504]; smaller values
      // keep 2^-24 absolute precision): the operand type of both attention
      // products, whose int8 keys and values convert to f16 by integer ops
      *reinterpret_cast<uint2*>(dst + d0) = make_uint2(pack_f16x2(bf16_round(r0[0]), bf16_round(r0[1])),
                                                       pack_f16x2(bf16_round(r0[2]), bf16_round(r0[3])));
      *reinterpret_cast<uint2*>(dst + d0 + 128) = make_uint2(pack_f16x2(bf16_round(r1[0]), bf16_round(r1[1])),
                                                             pack_f16x2(bf16_round(r1[2]), bf16_round(r1[3])));
    }
  }
  if (et == 0) stamp(ts, 12);
  // this CTA has read its buffer: the peer may push its next tile into it
  __syncwarp();
  if (lane == 0) mbar_arrive_peer(pair_done, peer);
  workers_publish(p, et, op == kOpQkv ? kCQkv : kCAct);
  ++pair_cnt;
  return true;
}

// ----------------------------------------------------- worker: attention ---
// Converts 16 quantized values (one 16-byte chunk of a key row) into bf16 (K)
// or f16 (V) and stores them into a 128-byte-swizzled tile.
// int8 -> f16 of 4 bytes by integer ops (exact): the bytes, offset to
// unsigned, become the low mantissa bytes of 1024 + u (f16 0x6400 | u), and
// one packed subtraction of 1152 leaves u - 128, the signed value.
__device__ __forceinline__ void i8x4_to_f16x4(uint32_t x, uint32_t& lo, uint32_t& hi) {
  x ^= 0x80808080u;
  const uint32_t a = __byte_perm(x, 0x64646464u, 0x4140);
  const uint32_t b = __byte_perm(x, 0x64646464u, 0x4342);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  const __half2 ra = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
  const __half2 rb = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
  lo = *reinterpret_cast<const uint32_t*>(&ra);
  hi = *reinterpret_cast<const uint32_t*>(&rb);
}

// 16 quantized values of one key (dims 16 g .. 16 g + 15) -> f16 into the
// K-major (K) or MN-major (V) swizzled tile: int8 values exactly (the key's
// scale is applied to its score / probability), uint8 values dequantized as
// the reference does, (u - zp) then * scale, each rounded to the scale dtype,
// then held as f16 (exact in f16's range).
__device__ __forceinline__ void convert16r(uint4 raw, uint8_t* tile_base, int key, int g, int mode, bool sbf16,
                                           float sc, float zp) {
  uint32_t w[8];
  if (mode == kQuantI8Sym) {
    i8x4_to_f16x4(raw.x, w[0], w[1]);
    i8x4_to_f16x4(raw.y, w[2], w[3]);
    i8x4_to_f16x4(raw.z, w[4], w[5]);
    i8x4_to_f16x4(raw.w, w[6], w[7]);
  } else {
    const uint8_t* b8 = reinterpret_cast<const uint8_t*>(&raw);
    float f[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float t = round_to(__fsub_rn(static_cast<float>(b8[e]), zp), sbf16);
      f[e] = round_to(__fmul_rn(t, sc), sbf16);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) w[e] = pack_f16x2(f[2 * e], f[2 * e + 1]);
  }
  uint8_t* atom = tile_base + (g >> 2) * 8192;
  const int c0 = (g & 3) * 2;
  *reinterpret_cast<uint4*>(atom + sw128_offset(key, c0)) = make_uint4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<uint4*>(atom + sw128_offset(key, c0 + 1)) = make_uint4(w[4], w[5], w[6], w[7]);
}

// Context-scheme instantiations of the attention worker: any scheme (read
// from the parameters) or int8 with fp32 scales fixed at compile time.  The
// fixed one is used for PI0, whose items walk 2-3 staged blocks each (its
// chunk 10.63 -> 10.38 ms); for PI0.5 (one block per item) the register
// allocation of the generic one came out 0.4 % faster.
constexpr int kScAny = 0, kScI8F32 = 1;

template <int V, bool DBG, int SC>
__device__ __forceinline__ bool worker_attn(const ChunkParams& p, uint8_t* smem, uint8_t* small, uint32_t tmem, int et, int layer,
                            unsigned use, int b, int qt, int sp, uint32_t& blk_cnt, uint32_t& kvn_cnt,
                            uint32_t& stg_cnt, unsigned long long* ts) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3;
  const int ch = et >> 7;  // this warp's half of the columns of its rows (S: 32 keys, O: 128 dims)
  uint8_t* sK = smem + kOffAK;
  uint8_t* sV = smem + kOffAV;
  uint8_t* sP = smem + kOffAP;
  // row maxima of the two column halves (two buffers, alternating by block)
  // and the final row sums, exchanged between the warps of a lane quadrant
  float* mx_x = reinterpret_cast<float*>(smem + kOffAXchg);  // [2][2][128]
  float* l_x = mx_x + 512;                                   // [2][128]
  uint64_t* conv_done = reinterpret_cast<uint64_t*>(small + kSmConv);
  uint64_t* s_full = reinterpret_cast<uint64_t*>(small + kSmSFull);
  uint64_t* p_ready = reinterpret_cast<uint64_t*>(small + kSmPReady);
  uint64_t* o_full = reinterpret_cast<uint64_t*>(small + kSmOFull);
  uint64_t* acc_free = reinterpret_cast<uint64_t*>(small + kSmAccFree);
  uint64_t* attn_done = reinterpret_cast<uint64_t*>(small + kSmAttnDone);
  uint64_t* kvn_full = reinterpret_cast<uint64_t*>(small + kSmKvnFull);
  uint64_t* stg_full = reinterpret_cast<uint64_t*>(small + kSmStgFull);
  uint64_t* stg_empty = reinterpret_cast<uint64_t*>(small + kSmStgEmpty);
  uint64_t* v_ready = reinterpret_cast<uint64_t*>(small + kSmVReady);
  const uint8_t* stg = smem + kOffAStg;
  const uint32_t tmO = tmem, tmS = tmem + 256;
  const int blk_begin = sp * p.n_blocks / p.attn_splits;
  const int nbl = (sp + 1) * p.n_blocks / p.attn_splits - blk_begin;
  const int r = quad * 32 + lane;
  const int R = qt * kQR + r;
  const bool row_valid = R < p.Hq * p.S;
  const int s_row = row_valid ? R % p.S : 0;
  const int h_row = row_valid ? R / p.S : 0;
  // block of this query row among the new tokens: new key j is visible iff
  // new_block[j] <= it (PI0's state token does not see the action tokens)
  const int my_block = (V == kPi0 && row_valid && p.new_block) ? p.new_block[s_row] : 0;
  const bool sbf16 = SC == kScI8F32 ? false : p.scale_bf16 != 0;
  const int mode = SC == kScI8F32 ? static_cast<int>(kQuantI8Sym) : p.mode;
  const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;
  bool new_ready = false;
  // per-key values of a block, in two sets alternating by block: [0, 64)
  // score scale (log2 units, 0 for a masked key), [64, 128) value scale,
  // [128, 192) additive mask, [192, 256) block ids of new keys (int), then
  // (uint8 scheme) K / V dequantization scales and K / V zero points
  auto scale_set = [&](int jl) { return reinterpret_cast<float*>(smem + ((jl & 1) ? kOffAScales1 : kOffAScales)); };
  // Block j's per-key values into set sc, in two halves: request() starts
  // the asynchronous copies of the per-key scales (fp32) and zero points of a
  // context block, finish() (after the copies of this thread completed)
  // turns them into the softmax's values; bf16 scales are loaded in finish().
  const bool async_sc = !sbf16;
  auto request = [&](int j, float* sc) {
    if (et >= 64 || j >= p.n_ctx_blocks || !async_sc) return;
    const long slot = static_cast<long>(j) * kKB + et;
    const long gi = static_cast<long>(b) * p.cap + (slot < p.cap ? slot : p.cap - 1);
    if (mode == kQuantI8Sym) {
      cp_async4(sc + et, static_cast<const float*>(p.k_scale[layer]) + gi);
      cp_async4(sc + 64 + et, static_cast<const float*>(p.v_scale[layer]) + gi);
    } else {
      cp_async4(sc + 256 + et, static_cast<const float*>(p.k_scale[layer]) + gi);
      cp_async4(sc + 320 + et, static_cast<const float*>(p.v_scale[layer]) + gi);
      cp_async4(sc + 384 + et, static_cast<const float*>(p.k_zp[layer]) + gi);
      cp_async4(sc + 448 + et, static_cast<const float*>(p.v_zp[layer]) + gi);
    }
    cp_async_commit();
  };
  auto finish = [&](int j, float* sc) {
    if (et >= 64) return;
    int* nb = reinterpret_cast<int*>(sc + 192);
    if (j < p.n_ctx_blocks) {
      const long slot = static_cast<long>(j) * kKB + et;
      const long gi = static_cast<long>(b) * p.cap + (slot < p.cap ? slot : p.cap - 1);
      const bool valid = slot < p.n_ctx && (!p.ctx_valid || p.ctx_valid[gi] != 0);
      if (async_sc) {
        cp_async_wait_all();
      } else {
        sc[256 + et] = load_scalar(p.k_scale[layer], gi, true);
        sc[320 + et] = load_scalar(p.v_scale[layer], gi, true);
        sc[384 + et] = load_scalar(p.k_zp[layer], gi, true);
        sc[448 + et] = load_scalar(p.v_zp[layer], gi, true);
      }
      if (mode == kQuantI8Sym) {
        sc[et] = valid ? sc[et] * p.scale_log2 : 0.f;
        sc[64 + et] = valid ? sc[64 + et] : 0.f;
      } else {
        sc[et] = valid ? p.scale_log2 : 0.f;
        sc[64 + et] = 1.f;
      }
      sc[128 + et] = valid ? 0.f : -INFINITY;
      nb[et] = 0;
    } else {
      const int kk = (j - p.n_ctx_blocks) * kKB + et;
      sc[et] = kk < p.S ? p.scale_log2 : 0.f;
      sc[64 + et] = 1.f;
      sc[128 + et] = kk < p.S ? 0.f : -INFINITY;
      nb[et] = (V == kPi0 && kk < p.S && p.new_block) ? p.new_block[kk] : 0;
    }
  };

  // ---- block pipeline.  Block jl: QK (MMA) -> softmax -> P; then the next
  // block's K is converted into sK (free once QK(jl) is done), so the MMA
  // issues QK(jl + 1) right after P.V(jl), and its V follows into sV once
  // P.V(jl) is done.  Iteration -1 prepares the first block. ----
  auto wait_all = [&](uint64_t* bar, uint32_t parity, int code) {
    bool w = true;
    if (lane == 0) w = bar_wait(p, bar, parity, code);
    return workers_all(__shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0);
  };
  // K (half 0) or V (half 1) of block j into sK / sV: the staged int8 rows
  // of a context block, or the new tokens' f16 rows
  auto fill = [&](int j, int half, const float* sc) {
    uint8_t* tile = half ? sV : sK;
    if (j < p.n_ctx_blocks) {
      const float* dq = sc + 256 + half * 64;
      const float* zq = sc + 384 + half * 64;
      const bool u8 = mode != kQuantI8Sym;
#pragma unroll 4
      for (int q = 0; q < 4; ++q) {
        const int it = et + q * kWorkers;  // 0..1023: 16 chunks of 16 bytes per key
        const int key = it >> 4, g = it & 15;
        const uint4 raw = *reinterpret_cast<const uint4*>(stg + half * kStgBytes + key * kD + g * 16);
        convert16r(raw, tile, key, g, mode, sbf16, u8 ? dq[key] : 0.f, u8 ? zq[key] : 0.f);
      }
    } else {
      const int nb0 = (j - p.n_ctx_blocks) * kKB;
      const __nv_bfloat16* rows = half ? p.vn : p.kn;
#pragma unroll 2
      for (int it = et; it < kKB * 32; it += kWorkers) {
        const int key = it >> 5, c = it & 31;
        const int kk = nb0 + key;
        uint4 raw = make_uint4(0u, 0u, 0u, 0u);
        if (kk < p.S) raw = __ldcg(reinterpret_cast<const uint4*>(rows + (static_cast<long>(b) * p.S + kk) * kD + c * 8));
        *reinterpret_cast<uint4*>(tile + (c >> 3) * 8192 + sw128_offset(key, c & 7)) = raw;
      }
    }
    fence_proxy_async_smem();
    workers_sync();
  };

  for (int jl = -1; jl < nbl && ok; ++jl) {
    const bool more = jl + 1 < nbl;
    if (jl >= 0) {
      const int j = blk_begin + jl;
      const bool causal = V == kPi0 && j >= p.n_ctx_blocks && p.new_block != nullptr;
      const float* sc = scale_set(jl);
      const float* ks_s = sc;
      const float* vs_s = sc + 64;
      const float* kadd_s = sc + 128;
      const int* nb_s = reinterpret_cast<const int*>(sc + 192);
      if (more) request(j + 1, scale_set(jl + 1));  // in flight during this block's softmax

      // ---- softmax on S ----
      if (!wait_all(s_full, blk_cnt & 1, kDevTimeoutMmaDone)) {
        ok = false;
        break;
      }
      ++blk_cnt;
      if (et == 0 && jl == 0) stamp(ts, 1);
      if (et == 0 && jl == 1) stamp(ts, 8);
      tc_fence_after();
      // two passes over this warp's 32 score columns in TMEM (16 at a time): the
      // block max (combined with the other column half through shared memory),
      // then p = 2^(z - m) -> P tile; scores in log2 units, one FMA per key
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int qq = 0; qq < 2; ++qq) {
        const int q = 2 * ch + qq;
        uint32_t rr[16];
        tmem_ld16(tmS + lane_base + q * 16, rr);
        tmem_wait_ld();
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = 4 * q + cc;
          const float4 km = reinterpret_cast<const float4*>(ks_s)[c];
          float4 ka = reinterpret_cast<const float4*>(kadd_s)[c];
          if (causal) {
            const int4 nb = reinterpret_cast<const int4*>(nb_s)[c];
            if (nb.x > my_block) ka.x = -INFINITY;
            if (nb.y > my_block) ka.y = -INFINITY;
            if (nb.z > my_block) ka.z = -INFINITY;
            if (nb.w > my_block) ka.w = -INFINITY;
          }
          mx[0] = fmaxf(mx[0], fmaf(__uint_as_float(rr[4 * cc + 0]), km.x, ka.x));
          mx[1] = fmaxf(mx[1], fmaf(__uint_as_float(rr[4 * cc + 1]), km.y, ka.y));
          mx[2] = fmaxf(mx[2], fmaf(__uint_as_float(rr[4 * cc + 2]), km.z, ka.z));
          mx[3] = fmaxf(mx[3], fmaf(__uint_as_float(rr[4 * cc + 3]), km.w, ka.w));
        }
      }
      float* mxb = mx_x + (jl & 1) * 256;
      mxb[ch * 128 + r] = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      quad_pair_sync(quad);
      const float bmax = fmaxf(mxb[r], mxb[128 + r]);
      const float m_new = fmaxf(m_run, bmax);
      bool need = false;
      float m_use;
      if (m_run == -INFINITY) {
        m_use = m_new;
      } else if (m_new > m_run + 8.f) {
        need = true;
        m_use = m_new;
      } else {
        m_use = m_run;
      }
      const float alpha = need ? exp2f(m_run - m_use) : 1.f;
      const float m_sub = m_use == -INFINITY ? 0.f : m_use;
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int qq = 0; qq < 2; ++qq) {
        const int q = 2 * ch + qq;
        uint32_t rr[16];
        tmem_ld16(tmS + lane_base + q * 16, rr);
        tmem_wait_ld();
        float pvq[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = 4 * q + cc;
          const float4 km = reinterpret_cast<const float4*>(ks_s)[c];
          float4 ka = reinterpret_cast<const float4*>(kadd_s)[c];
          if (causal) {
            const int4 nb = reinterpret_cast<const int4*>(nb_s)[c];
            if (nb.x > my_block) ka.x = -INFINITY;
            if (nb.y > my_block) ka.y = -INFINITY;
            if (nb.z > my_block) ka.z = -INFINITY;
            if (nb.w > my_block) ka.w = -INFINITY;
          }
          const float4 vsc = reinterpret_cast<const float4*>(vs_s)[c];
          const float zz[4] = {fmaf(__uint_as_float(rr[4 * cc + 0]), km.x, ka.x),
                               fmaf(__uint_as_float(rr[4 * cc + 1]), km.y, ka.y),
                               fmaf(__uint_as_float(rr[4 * cc + 2]), km.z, ka.z),
                               fmaf(__uint_as_float(rr[4 * cc + 3]), km.w, ka.w)};
          const float vv[4] = {vsc.x, vsc.y, vsc.z, vsc.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float pe = ex2_approx(zz[e] - m_sub);
            ps[e] += pe;
            pvq[4 * cc + e] = pe * vv[e];
          }
        }
        // keys 16q .. 16q+15 of row r: two 16-byte chunks of the P tile
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const uint4 v = make_uint4(pack_f16x2(pvq[8 * h2 + 0], pvq[8 * h2 + 1]),
                                     pack_f16x2(pvq[8 * h2 + 2], pvq[8 * h2 + 3]),
                                     pack_f16x2(pvq[8 * h2 + 4], pvq[8 * h2 + 5]),
                                     pack_f16x2(pvq[8 * h2 + 6], pvq[8 * h2 + 7]));
          *reinterpret_cast<uint4*>(sP + sw128_offset(r, 2 * q + h2)) = v;
        }
      }
      const float psum = (ps[0] + ps[1]) + (ps[2] + ps[3]);
      l_run = l_run * alpha + psum;
      m_run = m_use;
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c0 = 8 * ch; c0 < 8 * ch + 8; c0 += 2) {
          uint32_t rr[2][16];
#pragma unroll
          for (int q = 0; q < 2; ++q) tmem_ld16(tmO + lane_base + (c0 + q) * 16, rr[q]);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 2; ++q) {
#pragma unroll
            for (int e = 0; e < 16; ++e) rr[q][e] = __float_as_uint(__uint_as_float(rr[q][e]) * alpha);
            tmem_st16(tmO + lane_base + (c0 + q) * 16, rr[q]);
          }
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
      if (et == 0 && jl == 1) stamp(ts, 9);
    }
    if (!more) break;

    // ---- block jl + 1: per-key values, K, then (after P.V(jl)) V ----
    const int jn = blk_begin + jl + 1;
    float* scn = scale_set(jl + 1);
    if (jl < 0) request(jn, scn);
    finish(jn, scn);
    if (jn >= p.n_ctx_blocks && nbl == 1) {
      // the item's only block holds the new keys: the producer loads its K
      // and V tiles by TMA once the QKV tiles are published
      ok = wait_all(kvn_full, kvn_cnt & 1, kDevTimeoutTmaFull);  // also orders the values above
      ++kvn_cnt;
      if (ok && lane == 0) {
        mbar_arrive(conv_done);
        mbar_arrive(v_ready);
      }
      continue;
    }
    if (jn < p.n_ctx_blocks) {
      // the int8 rows, staged by the producer
      bool w = true;
      if (lane == 0) w = bar_wait(p, stg_full, stg_cnt & 1, kDevTimeoutTmaFull);
      w = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
      // every reader observes the completed phase itself (it completed for
      // lane 0, so this returns at once)
      for (int n = 0; w && lane != 0 && n < (1 << 16) && !mbar_try_wait(stg_full, stg_cnt & 1); ++n) {
      }
      ++stg_cnt;
      ok = workers_all(w);  // also orders the values above
    } else {
      // the new tokens' rows, written by this layer's QKV tiles
      if (!new_ready)
        ok = workers_ctr_wait(p, et, kCQkv,
                              static_cast<unsigned>(p.op[kOpQkv].m_tiles * p.op[kOpQkv].splits) * (use + 1));
      new_ready = true;
      if (ok) workers_sync();
    }
    if (!ok) break;
    fill(jn, 0, scn);
    if (lane == 0) mbar_arrive(conv_done);
    if (et == 0 && jl == 1) stamp(ts, 10);
    if (jl >= 0 && !wait_all(o_full, (blk_cnt - 1) & 1, kDevTimeoutMmaDone)) {
      ok = false;
      break;
    }
    if (et == 0 && jl == 1) stamp(ts, 11);
    fill(jn, 1, scn);
    if (lane == 0) mbar_arrive(v_ready);
    if (jn < p.n_ctx_blocks) {
      __syncwarp();
      if (lane == 0) mbar_arrive(stg_empty);  // this warp's share of the staging buffer is read
    }
    if (et == 0 && jl == -1) stamp(ts, 6);
    if (et == 0 && jl == 1) stamp(ts, 15);
  }

  // ---- epilogue: partial (O, m, l) of this split ----
  if (ok && nbl > 0) {
    bool w = true;
    if (lane == 0) w = bar_wait(p, o_full, (blk_cnt - 1) & 1, kDevTimeoutMmaDone);
    ok = workers_all(__shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0);
  }
  if (ok && nbl > 0) {
    if (et == 0) stamp(ts, 7);
    tc_fence_after();
    const long wcta = (static_cast<long>(b) * p.q_tiles + qt) * p.attn_splits + sp;
    const bool final_out = p.attn_splits == 1;
    l_x[ch * 128 + r] = l_run;
    quad_pair_sync(quad);
    l_run = l_x[r] + l_x[128 + r];
    const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
    const long tok = static_cast<long>(b) * p.S + s_row;
    __nv_bfloat16* orow = p.attn_out + tok * (static_cast<long>(p.Hq) * kD) + h_row * kD;
    // partial O of the split, normalized by its own l and kept as f16 (the
    // combine weights it by l * 2^(m - M)): [cta][16-column chunk][row][16]
    __half* wrow_o = reinterpret_cast<__half*>(p.ws_o) + (wcta * (kD / 16) * kQR + r) * 16;
#pragma unroll 1
    for (int c0 = 8 * ch; c0 < 8 * ch + 8; c0 += 4) {
      uint32_t rr[4][16];
#pragma unroll
      for (int q = 0; q < 4; ++q) tmem_ld16(tmO + lane_base + (c0 + q) * 16, rr[q]);
      tmem_wait_ld();
      if (!row_valid) continue;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int c = c0 + q;
        if (final_out) {
          uint32_t w8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            w8[e] = pack_bf16x2(__uint_as_float(rr[q][2 * e]) * inv_l, __uint_as_float(rr[q][2 * e + 1]) * inv_l);
          *reinterpret_cast<uint4*>(orow + c * 16) = make_uint4(w8[0], w8[1], w8[2], w8[3]);
          *reinterpret_cast<uint4*>(orow + c * 16 + 8) = make_uint4(w8[4], w8[5], w8[6], w8[7]);
          if (DBG && p.dbg_attn && use < static_cast<unsigned>(p.NL)) {
            __nv_bfloat16* drow = p.dbg_attn + static_cast<long>(use) * p.T * p.Hq * kD + (orow - p.attn_out);
            *reinterpret_cast<uint4*>(drow + c * 16) = make_uint4(w8[0], w8[1], w8[2], w8[3]);
            *reinterpret_cast<uint4*>(drow + c * 16 + 8) = make_uint4(w8[4], w8[5], w8[6], w8[7]);
          }
        } else {
          uint32_t w8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            w8[e] = pack_f16x2(__uint_as_float(rr[q][2 * e]) * inv_l, __uint_as_float(rr[q][2 * e + 1]) * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(wrow_o + static_cast<long>(c) * kQR * 16);
          __stcg(dst, make_uint4(w8[0], w8[1], w8[2], w8[3]));
          __stcg(dst + 1, make_uint4(w8[4], w8[5], w8[6], w8[7]));
        }
      }
    }
    if (!final_out && row_valid && ch == 0) __stcg(p.ws_ml + wcta * kQR + r, make_float2(m_run, l_run));
  }
  // TMEM and the ring's shared memory are free again
  tc_fence_before();
  __syncwarp();
  if (lane == 0) {
    mbar_arrive(acc_free);
    mbar_arrive(attn_done);
  }
  if (!ok) return false;
  workers_publish(p, et, kCAttn);
  return true;
}

// ------------------------------------------------------ worker: combine ---
template <bool DBG>
__device__ __forceinline__ bool worker_comb(const ChunkParams& p, uint8_t* smem, int et, unsigned use, int b, int qt,
                                            int r0, int r1, unsigned long long* ts) {
  if (!workers_ctr_wait(p, et, kCAttn, static_cast<unsigned>(p.n_attn) * (use + 1))) return false;
  if (et == 0) stamp(ts, 1);
  const int wq = et >> 5, lane = et & 31;
  // two warps per row (r1 - r0 <= 4 rows), each summing half of the splits;
  // the second half's sums meet the first's in the accumulator-tile buffer
  // (idle here: the paired tiles that fill it need this layer's combine)
  const int r = r0 + (wq & 3), half = wq >> 2;
  const int R = qt * kQR + r;
  const bool active = r < r1 && R < p.Hq * p.S;
  float* xchg = reinterpret_cast<float*>(smem + kOffRed) + ((wq & 3) * 32 + lane) * 8;
  constexpr int kBatch = 8;  // splits whose partials are in flight together
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float L = 0.f;
  if (active) {
    const long base = (static_cast<long>(b) * p.q_tiles + qt) * p.attn_splits;
    // lane: 8 of the row's 256 columns (chunk lane / 2, half lane % 2)
    const __half* ob = reinterpret_cast<const __half*>(p.ws_o) + ((lane >> 1) * kQR + r) * 16 + (lane & 1) * 8;
    const int s_mid = (p.attn_splits + 1) >> 1;
    const int s_begin = half ? s_mid : 0, s_end = half ? p.attn_splits : s_mid;
    // split s's (m, l) sits in lane s % 32, as the first (s < 32) or second
    // of its pair: the row max M and the weights w_s = l_s * 2^(m_s - M) are
    // warp reductions and broadcasts
    uint4 o[kBatch];
#pragma unroll
    for (int q = 0; q < kBatch; ++q)
      if (s_begin + q < s_end)
        o[q] = __ldcg(reinterpret_cast<const uint4*>(ob + (base + s_begin + q) * (kD / 16) * kQR * 16));
    const float2 ml = lane < p.attn_splits ? __ldcg(p.ws_ml + (base + lane) * kQR + r) : make_float2(-INFINITY, 0.f);
    const float2 ml2 =
        lane + 32 < p.attn_splits ? __ldcg(p.ws_ml + (base + lane + 32) * kQR + r) : make_float2(-INFINITY, 0.f);
    const bool live = ml.x != -INFINITY && ml.y > 0.f;
    const bool live2 = ml2.x != -INFINITY && ml2.y > 0.f;
    const float M = warp_max(fmaxf(live ? ml.x : -INFINITY, live2 ? ml2.x : -INFINITY));
    const float w = live ? exp2f(ml.x - M) * ml.y : 0.f;
    const float w2 = live2 ? exp2f(ml2.x - M) * ml2.y : 0.f;
    L = warp_sum(w + w2);
    for (int s0 = s_begin; s0 < s_end; s0 += kBatch) {
      if (s0 > s_begin) {
#pragma unroll
        for (int q = 0; q < kBatch; ++q)
          if (s0 + q < s_end) o[q] = __ldcg(reinterpret_cast<const uint4*>(ob + (base + s0 + q) * (kD / 16) * kQR * 16));
      }
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        const float ws = __shfl_sync(0xffffffffu, s0 + q < 32 ? w : w2, (s0 + q) & 31);
        if (s0 + q >= s_end) continue;
        const __half2* h2 = reinterpret_cast<const __half2*>(&o[q]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(h2[e]);
          acc[2 * e] = fmaf(ws, f.x, acc[2 * e]);
          acc[2 * e + 1] = fmaf(ws, f.y, acc[2 * e + 1]);
        }
      }
    }
    if (half) {
      *reinterpret_cast<float4*>(xchg) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(xchg + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
  workers_sync();
  if (active && !half) {
    const float4 u = *reinterpret_cast<const float4*>(xchg);
    const float4 v = *reinterpret_cast<const float4*>(xchg + 4);
    const float hsum[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
    const float inv = L > 0.f ? 1.f / L : 0.f;
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = (acc[e] + hsum[e]) * inv;
    const int s_row = R % p.S, h_row = R / p.S;
    __nv_bfloat16* orow =
        p.attn_out + (static_cast<long>(b) * p.S + s_row) * (static_cast<long>(p.Hq) * kD) + h_row * kD + lane * 8;
    const uint4 packed = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                                    pack_bf16x2(y[6], y[7]));
    *reinterpret_cast<uint4*>(orow) = packed;
    if (DBG && p.dbg_attn && use < static_cast<unsigned>(p.NL))
      *reinterpret_cast<uint4*>(p.dbg_attn + static_cast<long>(use) * p.T * p.Hq * kD + (orow - p.attn_out)) = packed;
  }
  workers_sync();  // the buffer is read before any later use of it
  workers_publish(p, et, kCComb);
  return true;
}

// PI0's per-step prefix of the token rows: the state token's projection and
// the action-time MLP (action_in_proj -> concat with the time embedding ->
// action_time_mlp_in -> SiLU -> action_time_mlp_out), reflex/policies/pi0/
// modeling_pi0.py embed_suffix.  Kept out of line so that its registers do not
// add to the PI0.5 finalize path.
__device__ __noinline__ bool worker_fin_at(const ChunkParams& p, uint8_t* small, int et, int kind, int tau, int t,
                                           unsigned long long* ts) {
  float* red8 = reinterpret_cast<float*>(small + kSmRed8);
  float* xs = reinterpret_cast<float*>(small + kSmXs);
  const int f0 = et * 4;
  const int b = t / p.S, s = t - b * p.S;
  const int sa = s - 1;         // action row of the token (-1: the state token)
  const int at = b * p.SA + sa;  // its row in the action-major buffers
  if (kind == kTInit) {
    float hv[4];
    if (sa < 0) {
      if (et < p.SD) xs[et] = bf16_round(p.state[static_cast<long>(b) * p.SD + et]);
      workers_sync();
      proj_in4(p, et, xs, hv, p.w_st, p.b_st, p.SD);
      *reinterpret_cast<uint2*>(p.st_emb + static_cast<long>(b) * p.W + f0) = pack4_bf16(hv);
    } else {
      if (et < p.A) xs[et] = bf16_round(p.x[static_cast<long>(at) * p.A + et]);
      workers_sync();
      action_in4(p, et, xs, hv);
      write_at_x(p, et, at, 0, hv);
    }
    workers_publish(p, et, kCAtX);
    return true;
  }
  if (kind == kTFinAt1 || kind == kTFinAt2) {
    const bool first = kind == kTFinAt1;
    const int op = first ? kOpAtIn : kOpAtOut;
    const OpCfg oc = op_cfg(p, op);
    NormVec nv1;
    if (!first) load_norm_vec(p, et, tau, 0, nv1);  // the first layer's input norm
    if (!workers_ctr_wait(p, et, first ? kCPat1 : kCPat2, static_cast<unsigned>(oc.m_tiles * oc.splits) * (tau + 1)))
      return false;
    if (et == 0) stamp(ts, 1);
    float hv[4];
    if (sa >= 0) {
      float acc[4];
      sum_partials4(p, op, at, f0, acc);
      const float4 bias = *reinterpret_cast<const float4*>((first ? p.b_atin : p.b_atout) + f0);
      const float bb[4] = {bias.x, bias.y, bias.z, bias.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v = bf16_round(acc[e] + bb[e]);
        hv[e] = first ? bf16_round(v / (1.f + expf(-v))) : v;
      }
      if (first) *reinterpret_cast<uint2*>(p.at_hid + static_cast<long>(at) * p.W + f0) = pack4_bf16(hv);
    } else if (!first) {
      unpack4_bf16(__ldcg(reinterpret_cast<const uint2*>(p.st_emb + static_cast<long>(b) * p.W + f0)), hv);
    }
    if (first) {
      workers_publish(p, et, kCAtH);
      return true;
    }
    *reinterpret_cast<uint2*>(p.h + static_cast<long>(t) * p.W + f0) = pack4_bf16(hv);
    float y[4];
    norm_row(p, et, hv, nv1, red8, y);
    *reinterpret_cast<uint2*>(p.xn + static_cast<long>(t) * p.W + f0) = pack4_bf16(y);
    workers_publish(p, et, kCXn);
    return true;
  }
  return false;
}

// ------------------------------------------ worker: per-token finalization ---
// kind kTInit: the first step's input (PI0.5: h = action_in_proj(x) and its
// norm; PI0: state_proj(state) for the state token, [action_in(x), t_emb]
// for the action tokens); kTFinO / kTFinD: the gated residual of o_proj /
// down_proj, then the next norm (or the Euler tail after the last layer);
// PI0's kTFinAt1 (action_time_mlp_in: bias + SiLU) and kTFinAt2
// (action_time_mlp_out: bias, or the state token's embedding, then the first
// layer's input norm).
template <int V, bool DBG>
__device__ __forceinline__ bool worker_fin(const ChunkParams& p, uint8_t* small, int et, int kind, int tau, int layer, int t,
                           unsigned long long* ts) {
  const int lane = et & 31, wq = et >> 5;
  float* red8 = reinterpret_cast<float*>(small + kSmRed8);
  // the tail's normalized row borrows the accumulator-tile buffer: the peer
  // CTA's next push into it belongs to a paired tile of the next Euler step,
  // whose input needs every tail of this step first
  float* row = reinterpret_cast<float*>(small - kOffSmall + kOffRed);
  float* xs = reinterpret_cast<float*>(small + kSmXs);
  const unsigned use = static_cast<unsigned>(tau * p.NL + layer);
  const int f0 = et * 4;
  const int b = t / p.S, s = t - b * p.S;
  constexpr bool pi0 = V == kPi0;
  const int sa = pi0 ? s - 1 : s;  // action row of the token (-1: PI0's state token)
  const int at = b * p.SA + sa;    // its row in the action-major buffers
  const bool tail = kind == kTFinD && layer == p.NL - 1;
  const bool next_step = tail && tau + 1 < p.steps;
  // everything that does not depend on the phase input is requested first
  NormVec nv1;
  const int n1 = kind == kTInit ? 0 : (kind == kTFinO ? 2 * layer + 1 : (tail ? 2 * p.NL : 2 * (layer + 1)));
  load_norm_vec(p, et, tau, n1, nv1);
  float g[4];
  if (kind != kTInit && p.gate) load4(p.gate + mod_off(p, tau, kind == kTFinO ? 2 * layer : 2 * layer + 1) + f0, g);
  float hv[4];
  if (kind == kTInit) {
    if (et < p.A) xs[et] = bf16_round(p.x[static_cast<long>(at) * p.A + et]);
    workers_sync();
    action_in4(p, et, xs, hv);
  } else {
    const int op = kind == kTFinO ? kOpO : kOpDown;
    const OpCfg oc = op_cfg(p, op);
    if (!workers_ctr_wait(p, et, kind == kTFinO ? kCPo : kCPd,
                          static_cast<unsigned>(oc.m_tiles * oc.splits) * (use + 1)))
      return false;
    if (et == 0) stamp(ts, 1);
    uint2 hraw = __ldcg(reinterpret_cast<const uint2*>(p.h + static_cast<long>(t) * p.W + f0));
    float acc[4];
    sum_partials4(p, op, t, f0, acc);
    float hres[4];
    unpack4_bf16(hraw, hres);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = bf16_round(acc[e]);
      const float ga = p.gate ? bf16_round(__fmul_rn(g[e], a)) : a;
      hv[e] = bf16_round(__fadd_rn(hres[e], ga));
    }
  }
  if (DBG && kind == kTFinD && tau == 0 && p.dbg_h)
    *reinterpret_cast<uint2*>(p.dbg_h + (static_cast<long>(layer) * p.T + t) * p.W + f0) = pack4_bf16(hv);
  if (tail) {
    if (sa < 0) {
      // PI0's state token: its next input row is rebuilt by kTFinAt2
      workers_publish(p, et, kCAtX);
      return true;
    }
    // final norm -> action_out_proj -> x += bf16(dt * v) -> next step's action_in_proj
    float y[4];
    norm_row(p, et, hv, nv1, red8, y);
#pragma unroll
    for (int e = 0; e < 4; ++e) row[f0 + e] = bf16_round(y[e]);
    workers_sync();
#pragma unroll 1
    for (int a = wq; a < p.A; a += kWorkers / 32) {
      const __nv_bfloat16* wr = p.w_out + static_cast<long>(a) * p.W;
      float acc = 0.f;
      for (int k = lane * 8; k < p.W; k += 256) {
        const uint4 raw = *reinterpret_cast<const uint4*>(wr + k);
        const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(w2[e]);
          acc = fmaf(f.x, row[k + 2 * e], acc);
          acc = fmaf(f.y, row[k + 2 * e + 1], acc);
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) {
        const float v = bf16_round(acc + (p.b_out ? __bfloat162float(p.b_out[a]) : 0.f));
        float* xp = p.x + static_cast<long>(at) * p.A + a;
        const float xn = __fadd_rn(*xp, bf16_round(__fmul_rn(p.dt, v)));
        *xp = xn;
        xs[a] = bf16_round(xn);
      }
    }
    workers_sync();
    if (!next_step) {
      workers_publish(p, et, pi0 ? kCAtX : kCXn);
      return true;
    }
    action_in4(p, et, xs, hv);
    if (pi0) {
      write_at_x(p, et, at, tau + 1, hv);
      workers_publish(p, et, kCAtX);
      return true;
    }
    load_norm_vec(p, et, tau + 1, 0, nv1);  // the next step's first input norm
  }
  *reinterpret_cast<uint2*>(p.h + static_cast<long>(t) * p.W + f0) = pack4_bf16(hv);
  float y[4];
  norm_row(p, et, hv, nv1, red8, y);
  *reinterpret_cast<uint2*>(p.xn + static_cast<long>(t) * p.W + f0) = pack4_bf16(y);
  workers_publish(p, et, (kind == kTFinO) ? kCXn2 : kCXn);
  return true;
}

// --------------------------------------------------------------- kernel ---
// Tensor maps of a GEMM op, selected with constant indices (a runtime index
// into the kernel parameters would copy them to local memory).
__device__ __forceinline__ const CUtensorMap* wmap(const Maps& maps, int op) {
  return op == kOpQkv ? &maps.w[kOpQkv] : op == kOpO ? &maps.w[kOpO] : op == kOpGu ? &maps.w[kOpGu]
         : op == kOpDown ? &maps.w[kOpDown] : op == kOpAtIn ? &maps.w[kOpAtIn] : &maps.w[kOpAtOut];
}
__device__ __forceinline__ const CUtensorMap* xmap(const Maps& maps, int op) {
  return op == kOpQkv ? &maps.x[kOpQkv] : op == kOpO ? &maps.x[kOpO] : op == kOpGu ? &maps.x[kOpGu]
         : op == kOpDown ? &maps.x[kOpDown] : op == kOpAtIn ? &maps.x[kOpAtIn] : &maps.x[kOpAtOut];
}

__device__ __forceinline__ int task_type(int4 t) { return t.x & 0xff; }
__device__ __forceinline__ int task_layer(int4 t) { return (t.x >> 8) & 0xff; }

// input counter of a GEMM op at use u
__device__ __forceinline__ void gemm_input(const ChunkParams& p, int op, unsigned use, int* line, unsigned* target) {
  switch (op) {
    case kOpQkv: *line = kCXn; *target = static_cast<unsigned>(p.n_fin) * (use + 1); break;
    case kOpO:
      if (p.attn_splits > 1) {
        *line = kCComb;
        *target = static_cast<unsigned>(p.n_comb) * (use + 1);
      } else {
        *line = kCAttn;
        *target = static_cast<unsigned>(p.n_attn) * (use + 1);
      }
      break;
    case kOpGu: *line = kCXn2; *target = static_cast<unsigned>(p.n_fin) * (use + 1); break;
    case kOpAtIn: *line = kCAtX; *target = static_cast<unsigned>(p.n_fin) * (use / p.NL + 1); break;
    case kOpAtOut: *line = kCAtH; *target = static_cast<unsigned>(p.n_fin) * (use / p.NL + 1); break;
    default:
      *line = kCAct;
      *target = static_cast<unsigned>(p.op[kOpGu].m_tiles * p.op[kOpGu].splits) * (use + 1);
      break;
  }
}

// V: kPi05 or kPi0 (PI0's code paths are compiled only into its instantiation);
// DBG: the instantiation that also writes the per-layer debug outputs
// (debug_hidden / debug_attn), kept out of the other one's loops; SC: the
// attention worker's context scheme (kScAny or kScI8F32)
template <int V, bool DBG, int SC>
__global__ void __launch_bounds__(kThreads, 1)
    chunk_kernel(const __grid_constant__ Maps maps, const __grid_constant__ ChunkParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* small = smem + kOffSmall;
  uint64_t* full = reinterpret_cast<uint64_t*>(small + kSmFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(small + kSmEmpty);
  uint64_t* acc_full = reinterpret_cast<uint64_t*>(small + kSmAccFull);
  uint64_t* acc_free = reinterpret_cast<uint64_t*>(small + kSmAccFree);
  uint64_t* q_full = reinterpret_cast<uint64_t*>(small + kSmQFull);
  uint64_t* conv_done = reinterpret_cast<uint64_t*>(small + kSmConv);
  uint64_t* s_full = reinterpret_cast<uint64_t*>(small + kSmSFull);
  uint64_t* p_ready = reinterpret_cast<uint64_t*>(small + kSmPReady);
  uint64_t* o_full = reinterpret_cast<uint64_t*>(small + kSmOFull);
  uint64_t* attn_done = reinterpret_cast<uint64_t*>(small + kSmAttnDone);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(small + kSmTmem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_free, kWorkers / 32);
    mbar_init(q_full, 1);
    mbar_init(conv_done, kWorkers / 32);
    mbar_init(s_full, 1);
    mbar_init(p_ready, kWorkers / 32);
    mbar_init(o_full, 1);
    mbar_init(attn_done, kWorkers / 32);
    mbar_init(reinterpret_cast<uint64_t*>(small + kSmKvnFull), 1);
    mbar_init(reinterpret_cast<uint64_t*>(small + kSmPairReady), kWorkers / 64);  // the peer's pushing warps
    mbar_init(reinterpret_cast<uint64_t*>(small + kSmPairDone), kWorkers / 32);
    mbar_init(reinterpret_cast<uint64_t*>(small + kSmMmaDrain), 1);
    mbar_init(reinterpret_cast<uint64_t*>(small + kSmStgFull), 1);
    mbar_init(reinterpret_cast<uint64_t*>(small + kSmStgEmpty), kWorkers / 32);
    mbar_init(reinterpret_cast<uint64_t*>(small + kSmVReady), kWorkers / 32);
    fence_mbar_init();
    for (int i = 0; i < (V == kPi0 ? kNumOps : kOpDown + 1); ++i) {
      tma_prefetch_desc(&maps.w[i]);
      tma_prefetch_desc(&maps.x[i]);
    }
    tma_prefetch_desc(&maps.q);
    tma_prefetch_desc(&maps.kn);
    tma_prefetch_desc(&maps.vn);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  cluster_sync();  // the peer CTA's barriers are initialized before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // modulation vectors and inputs of this chunk are written by earlier kernels

  const int cta = blockIdx.x;
  const int4* itasks = p.init_tasks + p.init_off[cta];
  const int n_init = p.init_off[cta + 1] - p.init_off[cta];
  const int4* stasks = p.step_tasks + p.step_off[cta];
  const int n_step = p.step_off[cta + 1] - p.step_off[cta];
  uint32_t issued = 0;  // ring stages issued by the producer
  uint32_t q_issued = 0, kvn_issued = 0;  // attention Q / new-key tile loads issued by the producer
  uint32_t stg_issued = 0;                // context blocks staged by the producer

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t attn_cnt = 0;
      bool ok = true;
      for (int tau = 0; tau < p.steps && ok; ++tau) {
        for (int i = 0; i < n_step && ok; ++i) {
          const int4 tk = stasks[i];
          const int ty = task_type(tk), layer = task_layer(tk);
          const unsigned use = static_cast<unsigned>(tau * p.NL + layer);
          if (gemm_op(ty) >= 0) {
            const int op = gemm_op(ty);
            const OpCfg oc = op_cfg(p, op);
            const int m = tk.y, kb0 = tk.w >> 16, kb1 = tk.w & 0xffff;
            const int nkb = kb1 - kb0;
            const int wrow = layer * oc.rows + m * kBM;
            const int nw = nkb < kStages ? nkb : kStages;
            int armed = 0;  // stages whose weight tile is in flight
            for (int j = 0; j < nw && ok; ++j) {
              const uint32_t ii = issued + j;
              const int s = ii % kStages;
              if (ii >= kStages) ok = bar_wait(p, &empty[s], ((ii / kStages) - 1) & 1, kDevTimeoutStageEmpty);
              if (!ok) break;
              mbar_arrive_expect_tx(&full[s], kWBytes + kXBytes);
              tma_load_2d_hint(smem + s * kWBytes, wmap(maps, op), &full[s], (kb0 + j) * kBK, wrow, pol);
              ++armed;
            }
            if (kTraceBuilt && p.trace && tau == 0 && i < p.trace_tasks)
              p.trace[(static_cast<long>(cta) * p.trace_tasks + i) * 16 + 7] = globaltimer_ns();
            int line;
            unsigned target;
            gemm_input(p, op, use, &line, &target);
            if (ok) ok = ctr_wait(p, line, target);
            if (kTraceBuilt && p.trace && tau == 0 && i < p.trace_tasks)
              p.trace[(static_cast<long>(cta) * p.trace_tasks + i) * 16 + 3] = globaltimer_ns();
            fence_proxy_async_global();
            // armed stages get their activation tile even after a failed wait,
            // so that every stage in flight completes and can be drained
            for (int j = 0; j < armed; ++j) {
              const int s = (issued + j) % kStages;
              tma_load_2d(smem + kOffX + s * kXBytes, xmap(maps, op), &full[s], (kb0 + j) * kBK, 0);
            }
            issued += armed;
            if (kTraceBuilt && p.trace && tau == 0 && i < p.trace_tasks && nw == nkb)
              p.trace[(static_cast<long>(cta) * p.trace_tasks + i) * 16 + 13] = globaltimer_ns();
            for (int j = nw; j < nkb && ok; ++j) {
              const uint32_t ii = issued;
              const int s = ii % kStages;
              ok = bar_wait(p, &empty[s], ((ii / kStages) - 1) & 1, kDevTimeoutStageEmpty);
              if (!ok) break;
              mbar_arrive_expect_tx(&full[s], kWBytes + kXBytes);
              tma_load_2d_hint(smem + s * kWBytes, wmap(maps, op), &full[s], (kb0 + j) * kBK, wrow, pol);
              tma_load_2d(smem + kOffX + s * kXBytes, xmap(maps, op), &full[s], (kb0 + j) * kBK, 0);
              ++issued;
            }
          } else if (ty == kTAttn) {
            // the ring's shared memory becomes the attention tiles: wait until
            // the MMA has consumed every stage issued so far
            for (uint32_t ii = (issued > kStages ? issued - kStages : 0); ii < issued && ok; ++ii)
              ok = bar_wait(p, &empty[ii % kStages], (ii / kStages) & 1, kDevTimeoutStageEmpty);
            if (!ok) break;
            unsigned long long* pts =
                (kTraceBuilt && p.trace && tau == 0 && i < p.trace_tasks) ? p.trace + (static_cast<long>(cta) * p.trace_tasks + i) * 16
                                                           : nullptr;
            stamp(pts, 12);
            const int b = tk.y, qt = tk.z;
            const int sp = tk.w;
            const int blk0 = sp * p.n_blocks / p.attn_splits;
            const int nbl = (sp + 1) * p.n_blocks / p.attn_splits - blk0;
            const int n_stage = max(0, min(nbl, p.n_ctx_blocks - blk0));  // context blocks of the item
            // context block j's int8 K / V rows (slots past the capacity are
            // not copied: those keys are masked and the stale bytes convert to
            // finite values) -> staging buffer, after the workers have
            // converted the block before it out of the buffer
            auto stage = [&](int j) {
              if (stg_issued > 0)
                ok = ok && bar_wait(p, reinterpret_cast<uint64_t*>(small + kSmStgEmpty), (stg_issued - 1) & 1,
                                    kDevTimeoutConvert);
              if (!ok) return;
              const int rows = min(kKB, p.cap - j * kKB);
              const uint32_t bytes = static_cast<uint32_t>(rows) * kD;
              const long off = (static_cast<long>(b) * p.cap + static_cast<long>(j) * kKB) * kD;
              uint64_t* stg_full = reinterpret_cast<uint64_t*>(small + kSmStgFull);
              mbar_arrive_expect_tx(stg_full, 2 * bytes);
              ++stg_issued;
              bulk_load(smem + kOffAStg, p.k_ring[layer] + off, bytes, stg_full);
              bulk_load(smem + kOffAStg + kStgBytes, p.v_ring[layer] + off, bytes, stg_full);
            };
            if (n_stage > 0) stage(blk0);
            if (!ok) break;
            ok = ctr_wait(p, kCQkv, static_cast<unsigned>(p.op[kOpQkv].m_tiles * p.op[kOpQkv].splits) * (use + 1));
            stamp(pts, 13);
            if (!ok) break;
            fence_proxy_async_global();
            const long q_row0 = static_cast<long>(b) * p.Hq * p.S + static_cast<long>(qt) * kQR;
            mbar_arrive_expect_tx(q_full, 4 * 16384);
            ++q_issued;
            for (int a = 0; a < 4; ++a)
              tma_load_2d(smem + kOffAQ + a * 16384, &maps.q, q_full, a * 64, static_cast<int>(q_row0));
            if (nbl == 1 && blk0 >= p.n_ctx_blocks) {
              // the new keys' K / V tiles (rows of the next stream, or zero
              // fill, beyond S are masked in the softmax)
              const int row0 = b * p.S + (blk0 - p.n_ctx_blocks) * kKB;
              uint64_t* kvn_full = reinterpret_cast<uint64_t*>(small + kSmKvnFull);
              mbar_arrive_expect_tx(kvn_full, 8 * 8192);
              ++kvn_issued;
              for (int a = 0; a < 4; ++a) {
                tma_load_2d(smem + kOffAK + a * 8192, &maps.kn, kvn_full, a * 64, row0);
                tma_load_2d(smem + kOffAV + a * 8192, &maps.vn, kvn_full, a * 64, row0);
              }
            }
            for (int jl = 1; jl < n_stage && ok; ++jl) stage(blk0 + jl);
            if (!ok) break;
            ok = bar_wait(p, attn_done, attn_cnt & 1, kDevTimeoutConvert);
            ++attn_cnt;
          }
        }
      }
      if (!ok) raise_abort(p, kDevTimeoutStageEmpty);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_g = make_idesc_f16(kBM, kNT, true);
      constexpr uint32_t idesc_s = make_idesc_f16(kQR, kKB, false);  // f16 Q and K
      constexpr uint32_t idesc_o = make_idesc_f16(kQR, kD, false, true);
      uint32_t consumed = 0, tmem_uses = 0, q_cnt = 0, conv_cnt = 0, p_cnt = 0;
      // ring stage 0's operand descriptors (shared-memory addresses stay below
      // 256 KB, so start-address offsets never carry out of their field)
      const uint64_t a_desc0 = make_sdesc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t b_desc0 = make_sdesc_sw128(smem_u32(smem + kOffX), 16, 1024);
      bool ok = true;
      for (int tau = 0; tau < p.steps && ok; ++tau) {
        for (int i = 0; i < n_step && ok; ++i) {
          const int4 tk = stasks[i];
          const int ty = task_type(tk);
          if (gemm_op(ty) >= 0) {
            const int nkb = (tk.w & 0xffff) - (tk.w >> 16);
            if (tmem_uses > 0) ok = bar_wait(p, acc_free, (tmem_uses - 1) & 1, kDevTimeoutMmaDone);
            if (!ok) break;
            ++tmem_uses;
            tc_fence_after();
            unsigned long long* mts =
                (kTraceBuilt && p.trace && tau == 0 && i < p.trace_tasks) ? p.trace + (static_cast<long>(cta) * p.trace_tasks + i) * 16
                                                           : nullptr;
            unsigned long long waited = 0;
            for (int j = 0; j < nkb && ok; ++j) {
              const uint32_t ii = consumed + j;
              const int s = ii % kStages;
              if (!mbar_try_wait(&full[s], (ii / kStages) & 1)) {
                const unsigned long long w0 = mts ? globaltimer_ns() : 0ull;
                ok = bar_wait(p, &full[s], (ii / kStages) & 1, kDevTimeoutTmaFull);
                if (mts && j > 0) waited += globaltimer_ns() - w0;
              }
              if (!ok) break;
              if (j == 0) stamp(mts, 10);
              if (j == nkb - 1) stamp(mts, 11);
              tc_fence_after();
              // descriptors of stage s: the base descriptors plus the stage's
              // byte offset >> 4 in the start-address field
              const uint64_t ad = a_desc0 + static_cast<uint64_t>((s * kWBytes) >> 4);
              const uint64_t bd = b_desc0 + static_cast<uint64_t>((s * kXBytes) >> 4);
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk)
                umma_f16_ss(tmem, ad + static_cast<uint64_t>(kk * 2), bd + static_cast<uint64_t>(kk * 2), idesc_g,
                            (j > 0 || kk > 0) ? 1u : 0u);
              umma_commit(&empty[s]);
            }
            consumed += nkb;
            if (mts) mts[14] = waited;
            if (ok) umma_commit(acc_full);
          } else if (ty == kTAttn) {
            const int sp = tk.w;
            const int blk_begin = sp * p.n_blocks / p.attn_splits;
            const int nbl = (sp + 1) * p.n_blocks / p.attn_splits - blk_begin;
            if (tmem_uses > 0) ok = bar_wait(p, acc_free, (tmem_uses - 1) & 1, kDevTimeoutMmaDone);
            if (!ok) break;
            ++tmem_uses;
            ok = bar_wait(p, q_full, q_cnt & 1, kDevTimeoutTmaFull);
            ++q_cnt;
            unsigned long long* mts =
                (kTraceBuilt && p.trace && tau == 0 && i < p.trace_tasks) ? p.trace + (static_cast<long>(cta) * p.trace_tasks + i) * 16
                                                           : nullptr;
            stamp(mts, 14);
            for (int jl = 0; jl < nbl && ok; ++jl) {
              ok = bar_wait(p, conv_done, conv_cnt & 1, kDevTimeoutConvert);
              ++conv_cnt;
              if (!ok) break;
              tc_fence_after();
#pragma unroll
              for (int ks = 0; ks < kD / 16; ++ks) {
                const int a = ks >> 2, kk = ks & 3;
                const uint64_t ad = make_sdesc_sw128(smem_u32(smem + kOffAQ + a * 16384) + kk * 32, 16, 1024);
                const uint64_t bd = make_sdesc_sw128(smem_u32(smem + kOffAK + a * 8192) + kk * 32, 16, 1024);
                umma_f16_ss(tmem + 256, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
              }
              umma_commit(s_full);
              ok = bar_wait(p, p_ready, p_cnt & 1, kDevTimeoutConvert) &&
                   bar_wait(p, reinterpret_cast<uint64_t*>(small + kSmVReady), p_cnt & 1, kDevTimeoutConvert);
              ++p_cnt;
              if (!ok) break;
              tc_fence_after();
#pragma unroll
              for (int ks = 0; ks < kKB / 16; ++ks) {
                const uint64_t ad = make_sdesc_sw128(smem_u32(smem + kOffAP) + ks * 32, 16, 1024);
                const uint64_t bd = make_sdesc_sw128(smem_u32(smem + kOffAV) + ks * 2048, 8192, 1024);
                umma_f16_ss(tmem, ad, bd, idesc_o, (jl > 0 || ks > 0) ? 1u : 0u);
              }
              umma_commit(o_full);
            }
          }
        }
      }
    }
  } else {
    const int et = threadIdx.x - 64;
    uint32_t acc_cnt = 0, blk_cnt = 0, kvn_cnt = 0, pair_cnt = 0, stg_cnt = 0;
    bool ok = true;
    for (int i = 0; i < n_init && ok; ++i)
      ok = V == kPi0 ? worker_fin_at(p, small, et, kTInit, 0, itasks[i].y, nullptr)
                     : worker_fin<V, DBG>(p, small, et, kTInit, 0, 0, itasks[i].y, nullptr);
    for (int tau = 0; tau < p.steps && ok; ++tau) {
      for (int i = 0; i < n_step && ok; ++i) {
        const int4 tk = stasks[i];
        const int ty = task_type(tk), layer = task_layer(tk);
        const unsigned use = static_cast<unsigned>(tau * p.NL + layer);
        unsigned long long* ts =
            (kTraceBuilt && p.trace && tau == 0 && i < p.trace_tasks) ? p.trace + (static_cast<long>(cta) * p.trace_tasks + i) * 16
                                                       : nullptr;
        if (et == 0) {
          stamp(ts, 0);
          if (ts) {
            ts[4] = static_cast<unsigned long long>(static_cast<unsigned>(tk.x)) |
                    (static_cast<unsigned long long>(static_cast<unsigned>(tk.y)) << 32);
            ts[5] = static_cast<unsigned long long>(static_cast<unsigned>(tk.z)) |
                    (static_cast<unsigned long long>(static_cast<unsigned>(tk.w)) << 32);
          }
        }
        switch (ty) {
          case kTQkv: case kTO: case kTGu: case kTDown: case kTAtIn: case kTAtOut:
            ok = worker_gemm(p, smem, small, tmem, et, gemm_op(ty), layer, tk.y, tk.z, acc_cnt, pair_cnt, ts);
            break;
          case kTAttn:
            ok = worker_attn<V, DBG, SC>(p, smem, small, tmem, et, layer, use, tk.y, tk.z, tk.w, blk_cnt, kvn_cnt, stg_cnt, ts);
            break;
          case kTComb: ok = worker_comb<DBG>(p, smem, et, use, tk.y, tk.z, tk.w >> 16, tk.w & 0xffff, ts); break;
          case kTFinO: case kTFinD: ok = worker_fin<V, DBG>(p, small, et, ty, tau, layer, tk.y, ts); break;
          case kTFinAt1: case kTFinAt2:
            if (V == kPi0) ok = worker_fin_at(p, small, et, ty, tau, tk.y, ts);
            break;
          default: break;
        }
        if (et == 0) stamp(ts, 2);
      }
    }
  }

  // ---- teardown: bounded drain of copies and MMAs in flight (after an
  // abort some were never waited for), then free TMEM ----
  __syncthreads();
  if (warp == 0 && lane == 0) {
    for (uint32_t ii = (issued > kStages ? issued - kStages : 0); ii < issued; ++ii)
      mbar_wait(&full[ii % kStages], (ii / kStages) & 1, p.status, kDevTimeoutTmaFull);
    if (q_issued > 0) mbar_wait(q_full, (q_issued - 1) & 1, p.status, kDevTimeoutTmaFull);
    if (kvn_issued > 0)
      mbar_wait(reinterpret_cast<uint64_t*>(small + kSmKvnFull), (kvn_issued - 1) & 1, p.status, kDevTimeoutTmaFull);
    if (stg_issued > 0)
      mbar_wait(reinterpret_cast<uint64_t*>(small + kSmStgFull), (stg_issued - 1) & 1, p.status, kDevTimeoutTmaFull);
  }
  if (warp == 1 && lane == 0) {
    uint64_t* drain = reinterpret_cast<uint64_t*>(small + kSmMmaDrain);
    umma_commit(drain);  // arrives once every MMA issued before it has completed
    mbar_wait(drain, 0, p.status, kDevTimeoutMmaDone);
  }
  // the peer CTA writes into this CTA's shared memory until its last paired item
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace
}  // namespace rfx

// ================================================================= host ===
namespace rfx {
namespace {

// QKV and gate/up tiles are split in two along K over the two CTAs of a
// cluster (summed through DSMEM); o_proj / down_proj tiles are split eight
// ways and summed per token by the next phase
constexpr int kSplitsQkv = 2, kSplitsO = 8, kSplitsGu = 2, kSplitsDown = 8;
constexpr int kMaxSplits = 64;  // attention key-range splits (the combine holds two per lane)

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// The executor instantiation of a variant, with or without the debug outputs.
using ChunkFn = void (*)(const Maps, const ChunkParams);
ChunkFn chunk_fn(int variant, bool dbg, bool i8_f32) {
  if (variant == kPi0) {
    if (i8_f32) return dbg ? chunk_kernel<kPi0, true, kScI8F32> : chunk_kernel<kPi0, false, kScI8F32>;
    return dbg ? chunk_kernel<kPi0, true, kScAny> : chunk_kernel<kPi0, false, kScAny>;
  }
  return dbg ? chunk_kernel<kPi05, true, kScAny> : chunk_kernel<kPi05, false, kScAny>;
}

struct Layout {
  int T, S, q_tiles, n_ctx_blocks, n_blocks, splits, n_attn, n_comb;
  OpCfg op[kNumOps];
  size_t off_ctr, off_part[kNumOps], off_ws_o, off_ws_ml, off_h, off_xn, off_q, off_kn, off_vn, off_attn, off_act,
      off_at_x, off_at_hid, off_st, off_ptrs, off_tasks, total;
};

// tokens per stream inside the layers: PI0 puts its state token first
int layer_tokens(const rfx_chunk_desc& d) { return d.S + (d.variant == RFX_CHUNK_PI0 ? 1 : 0); }

int validate(const rfx_chunk_desc& d) {
  if (d.variant != RFX_CHUNK_PI05 && d.variant != RFX_CHUNK_PI0) return set_error(RFX_E_INVAL, "rfx_chunk: variant");
  const int T = d.B * layer_tokens(d);
  if (d.B < 1 || d.S < 1 || T > kNT || d.num_layers < 1 || d.num_layers > 255 || d.num_steps < 1 ||
      d.width != 1024 || d.num_q_heads < 1 || (d.num_q_heads + 2) * 256 % kBM || d.mlp_dim < kBM ||
      d.mlp_dim % 64 || d.action_dim < 8 || d.action_dim > 64 || d.action_dim % 8)
    return set_error(RFX_E_UNSUPPORTED,
                     "rfx_chunk: needs B*S <= 64 tokens (PI0: B*(S+1)), width 1024, head_dim 256, mlp_dim %% 64 == 0, "
                     "action_dim 8..64 (multiple of 8)");
  if (d.variant == RFX_CHUNK_PI0 &&
      (!d.state || !d.w_state || !d.w_atin || !d.b_atin || !d.w_atout || !d.b_atout || !d.time_emb || !d.new_block ||
       d.state_dim < 8 || d.state_dim > 64 || d.state_dim % 8))
    return set_error(RFX_E_INVAL, "rfx_chunk: PI0 needs state, state_proj, action-time MLP, time embedding and "
                                  "new_block, state_dim 8..64 (multiple of 8)");
  if (!d.w_qkv || !d.w_o || !d.w_gu || !d.w_down || !d.norm_a1 || !d.w_in || !d.w_out || !d.rope_table ||
      !d.positions || !d.x || !d.k_ring || !d.v_ring || !d.k_scale || !d.v_scale)
    return set_error(RFX_E_INVAL, "rfx_chunk: null pointer in the descriptor");
  if (d.quant_mode != RFX_QUANT_I8_SYM && d.quant_mode != RFX_QUANT_U8_REF)
    return set_error(RFX_E_INVAL, "rfx_chunk: quant_mode");
  if (d.quant_mode == RFX_QUANT_I8_SYM && d.scale_dtype != RFX_DTYPE_F32)
    return set_error(RFX_E_INVAL, "rfx_chunk: the int8 scheme keeps fp32 scales");
  if (d.quant_mode == RFX_QUANT_U8_REF && (!d.k_zp || !d.v_zp))
    return set_error(RFX_E_INVAL, "rfx_chunk: the uint8 scheme needs zero points");
  if (d.n_ctx < 0 || d.capacity < 1 || d.n_ctx > d.capacity) return set_error(RFX_E_INVAL, "rfx_chunk: 0 <= n_ctx <= capacity");
  for (int l = 0; l < d.num_layers; ++l)
    if (!d.k_ring[l] || !d.v_ring[l] || !d.k_scale[l] || !d.v_scale[l] ||
        (d.quant_mode == RFX_QUANT_U8_REF && (!d.k_zp[l] || !d.v_zp[l])))
      return set_error(RFX_E_INVAL, "rfx_chunk: null ring pointer of layer %d", l);
  for (int l = 0; l < d.num_layers; ++l)  // context blocks are staged by bulk copies
    if ((reinterpret_cast<uintptr_t>(d.k_ring[l]) | reinterpret_cast<uintptr_t>(d.v_ring[l])) & 15)
      return set_error(RFX_E_INVAL, "rfx_chunk: the rings of layer %d must be 16-byte aligned", l);
  return RFX_OK;
}

Layout layout(const rfx_chunk_desc& d, int nct) {
  Layout L{};
  L.S = layer_tokens(d);
  L.T = d.B * L.S;
  const int hq = d.num_q_heads;
  const bool pi0 = d.variant == RFX_CHUNK_PI0;
  L.q_tiles = (hq * L.S + kQR - 1) / kQR;
  L.n_ctx_blocks = (d.n_ctx + kKB - 1) / kKB;
  L.n_blocks = L.n_ctx_blocks + (L.S + kKB - 1) / kKB;
  // by default one key block per split, or, for long contexts, as many
  // splits as put one attention item on each CTA (those without a QKV tile
  // take theirs first: they stage and convert their first block while the
  // QKV tiles run)
  int splits = d.kv_splits;
  if (splits <= 0) splits = std::max(1, nct / (d.B * L.q_tiles));
  splits = std::max(1, std::min({splits, L.n_blocks, kMaxSplits}));
  L.splits = splits;
  L.n_attn = d.B * L.q_tiles * splits;
  L.n_comb = splits > 1 ? d.B * L.q_tiles * (kQR / 4) : 0;  // 4 query rows (one per worker warp) per item
  const int rows[kNumOps] = {(hq + 2) * 256, d.width, 2 * d.mlp_dim, d.width, d.width, d.width};
  const int Ks[kNumOps] = {d.width, hq * 256, d.width, d.mlp_dim, 2 * d.width, d.width};
  const int sp[kNumOps] = {kSplitsQkv, kSplitsO, kSplitsGu, kSplitsDown, kSplitsO, kSplitsO};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  L.off_ctr = take(static_cast<size_t>(kNumCtrLines) * 128);
  for (int i = 0; i < kNumOps; ++i) {
    OpCfg& oc = L.op[i];
    oc.rows = rows[i];
    oc.K = Ks[i];
    oc.m_tiles = rows[i] / kBM;
    const int kb_total = Ks[i] / kBK;
    oc.splits = std::min(sp[i], kb_total);
    while (kb_total % oc.splits) --oc.splits;
    oc.kb = kb_total / oc.splits;
    const bool used = i <= kOpDown || pi0;  // PI0's action-time MLP
    L.off_part[i] = take(used ? static_cast<size_t>(oc.m_tiles) * oc.splits * kNT * kBM * 4 : 0);
  }
  const size_t wrows = static_cast<size_t>(d.B) * L.q_tiles * splits * kQR;
  L.off_ws_o = take(wrows * kD * 4);
  L.off_ws_ml = take(wrows * 8);
  L.off_h = take(static_cast<size_t>(L.T) * d.width * 2);
  L.off_xn = take(static_cast<size_t>(L.T) * d.width * 2);
  L.off_q = take(static_cast<size_t>(d.B) * hq * L.S * 256 * 2);
  L.off_kn = take(static_cast<size_t>(L.T) * 256 * 2);
  L.off_vn = take(static_cast<size_t>(L.T) * 256 * 2);
  L.off_attn = take(static_cast<size_t>(L.T) * hq * 256 * 2);
  L.off_act = take(static_cast<size_t>(L.T) * d.mlp_dim * 2);
  const size_t TA = static_cast<size_t>(d.B) * d.S;
  L.off_at_x = take(pi0 ? TA * 2 * d.width * 2 : 0);
  L.off_at_hid = take(pi0 ? TA * d.width * 2 : 0);
  L.off_st = take(pi0 ? static_cast<size_t>(d.B) * d.width * 2 : 0);
  L.off_ptrs = take(static_cast<size_t>(6) * d.num_layers * sizeof(void*));
  L.off_tasks = off;  // the task tables follow (size known after scheduling)
  L.total = off;
  return L;
}

struct Schedule {
  std::vector<int4> step, init;
  std::vector<int> step_off, init_off;
};

// Static task lists of every CTA, in phase order.  GEMM tiles go to the CTAs
// with the fewest items of the phase, then the fewest weight bytes so far, so
// the weight stream is spread over all SMs; attention items go to CTAs that
// take no o_proj tile in that layer (their shared memory is busy meanwhile).
Schedule build_schedule(const rfx_chunk_desc& d, const Layout& L, int nct) {
  std::vector<std::vector<int4>> lst(nct), ini(nct);
  std::vector<long> load(nct, 0);
  int rr = 0;  // rotating start for the light tasks
  auto enc = [](int type, int layer) { return type | (layer << 8); };
  auto task_of = [](int op) { return op <= kOpDown ? kTQkv + op : op == kOpAtIn ? kTAtIn : kTAtOut; };
  auto gemm_phase = [&](int layer, int op, const std::vector<char>& excl) {
    const OpCfg& oc = L.op[op];
    std::vector<int> cnt(nct, 0);
    std::vector<char> used(nct, 0);
    if (op == kOpQkv || op == kOpGu) {
      // split s of tile m on CTA rank s of one cluster; both CTAs of the
      // cluster get their tiles in the same order
      for (int m = 0; m < oc.m_tiles; ++m) {
        int best = -1;
        for (int c = 0; c + 1 < nct; c += 2) {
          if (excl[c] || excl[c + 1]) continue;
          const long lc = load[c] + load[c + 1], lb = best < 0 ? 0 : load[best] + load[best + 1];
          if (best < 0 || cnt[c] < cnt[best] || (cnt[c] == cnt[best] && lc < lb)) best = c;
        }
        for (int s = 0; s < 2; ++s) {
          const int kb0 = s * oc.kb, kb1 = kb0 + oc.kb;
          lst[best + s].push_back(make_int4(enc(task_of(op), layer), m, s, (kb0 << 16) | kb1));
          cnt[best + s]++;
          used[best + s] = 1;
          load[best + s] += static_cast<long>(oc.kb) * kWBytes;
        }
      }
      return used;
    }
    for (int m = 0; m < oc.m_tiles; ++m)
      for (int s = 0; s < oc.splits; ++s) {
        int best = -1;
        for (int c = 0; c < nct; ++c) {
          if (excl[c]) continue;
          if (best < 0 || cnt[c] < cnt[best] || (cnt[c] == cnt[best] && load[c] < load[best])) best = c;
        }
        const int kb0 = s * oc.kb, kb1 = kb0 + oc.kb;
        lst[best].push_back(make_int4(enc(task_of(op), layer), m, s, (kb0 << 16) | kb1));
        cnt[best]++;
        used[best] = 1;
        load[best] += static_cast<long>(oc.kb) * kWBytes;
      }
    return used;
  };
  auto light = [&](int4 t) {
    lst[rr % nct].push_back(t);
    ++rr;
  };
  for (int t = 0; t < L.T; ++t) ini[t % nct].push_back(make_int4(kTInit, t, 0, 0));
  const std::vector<char> none(nct, 0);
  if (d.variant == RFX_CHUNK_PI0) {
    // every step starts with the action-time MLP: [action_in(x), t_emb] ->
    // Linear + SiLU -> Linear -> the action rows of h (the state row is its
    // embedding), then the first layer's input norm
    gemm_phase(0, kOpAtIn, none);
    for (int t = 0; t < L.T; ++t) light(make_int4(enc(kTFinAt1, 0), t, 0, 0));
    gemm_phase(0, kOpAtOut, none);
    for (int t = 0; t < L.T; ++t) light(make_int4(enc(kTFinAt2, 0), t, 0, 0));
  }
  for (int l = 0; l < d.num_layers; ++l) {
    const std::vector<char> qkv_cta = gemm_phase(l, kOpQkv, none);
    // attention items go to CTAs without a QKV tile in this layer first, so
    // they stage and convert their first context block while the QKV tiles run
    std::vector<char> attn_cta(nct, 0);
    std::vector<int> order;  // CTAs without a QKV tile first, then the others
    for (int pass = 0; pass < 2; ++pass)
      for (int k = 0; k < nct; ++k) {
        const int c = (rr + k) % nct;
        if ((qkv_cta[c] != 0) == (pass == 1)) order.push_back(c);
      }
    int n_items = 0;
    for (int b = 0; b < d.B; ++b)
      for (int qt = 0; qt < L.q_tiles; ++qt)
        for (int s = 0; s < L.splits; ++s) {
          const int c = order[n_items++ % nct];
          attn_cta[c] = 1;
          lst[c].push_back(make_int4(enc(kTAttn, l), b, qt, s));
        }
    rr = order[n_items % nct];
    if (L.splits > 1)
      for (int b = 0; b < d.B; ++b)
        for (int qt = 0; qt < L.q_tiles; ++qt)
          for (int g = 0; g < kQR / 4; ++g) light(make_int4(enc(kTComb, l), b, qt, ((g * 4) << 16) | (g * 4 + 4)));
    // o_proj tiles avoid the attention CTAs (whose shared memory holds the
    // attention tiles until their item ends) when the others can take one
    // tile each
    int n_attn_cta = 0;
    for (char c : attn_cta) n_attn_cta += c;
    gemm_phase(l, kOpO, nct - n_attn_cta >= L.op[kOpO].m_tiles * L.op[kOpO].splits ? attn_cta : none);
    for (int t = 0; t < L.T; ++t) light(make_int4(enc(kTFinO, l), t, 0, 0));
    gemm_phase(l, kOpGu, none);
    gemm_phase(l, kOpDown, none);
    for (int t = 0; t < L.T; ++t) light(make_int4(enc(kTFinD, l), t, 0, 0));
  }
  Schedule S;
  S.step_off.push_back(0);
  S.init_off.push_back(0);
  for (int c = 0; c < nct; ++c) {
    S.step.insert(S.step.end(), lst[c].begin(), lst[c].end());
    S.step_off.push_back(static_cast<int>(S.step.size()));
    S.init.insert(S.init.end(), ini[c].begin(), ini[c].end());
    S.init_off.push_back(static_cast<int>(S.init.size()));
  }
  return S;
}

size_t schedule_bytes(const Schedule& s) {
  return align256(s.step.size() * sizeof(int4)) + align256(s.init.size() * sizeof(int4)) +
         align256(s.step_off.size() * sizeof(int)) + align256(s.init_off.size() * sizeof(int));
}

int chunk_grid() {
  int n = 148;
  rfx_num_sms(&n);
  return n & ~1;  // CTA pairs (clusters of two)
}

}  // namespace
}  // namespace rfx

struct rfx_chunk {
  rfx::Maps maps;
  rfx::ChunkParams params;
  size_t ctr_bytes = 0;
  int grid = 0;
  int max_tasks = 0;  // longest per-CTA task list of one step
  int device = -1;
};

extern "C" int rfx_chunk_workspace_size(const rfx_chunk_desc* desc, size_t* bytes) {
  using namespace rfx;
  if (!desc || !bytes) return set_error(RFX_E_INVAL, "rfx_chunk_workspace_size: null argument");
  int rc = validate(*desc);
  if (rc) return rc;
  const int nct = chunk_grid();
  const Layout L = layout(*desc, nct);
  *bytes = L.total + schedule_bytes(build_schedule(*desc, L, nct));
  return RFX_OK;
}

extern "C" int rfx_chunk_create(const rfx_chunk_desc* desc, void* workspace, size_t workspace_bytes,
                                rfx_chunk** out) {
  using namespace rfx;
  if (!desc || !out) return set_error(RFX_E_INVAL, "rfx_chunk_create: null argument");
  *out = nullptr;
  const rfx_chunk_desc& d = *desc;
  int rc = validate(d);
  if (rc) return rc;
  const int nct = chunk_grid();
  const Layout L = layout(d, nct);
  const Schedule S = build_schedule(d, L, nct);
  const size_t need = L.total + schedule_bytes(S);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return set_error(RFX_E_INVAL, "rfx_chunk_create: workspace of %zu bytes (256-byte aligned) required", need);
  char* ws = static_cast<char*>(workspace);

  auto* c = new (std::nothrow) rfx_chunk();
  if (!c) return set_error(RFX_E_INVAL, "rfx_chunk_create: out of host memory");
  cudaGetDevice(&c->device);
  c->grid = nct;
  for (int i = 0; i < nct; ++i) c->max_tasks = std::max(c->max_tasks, S.step_off[i + 1] - S.step_off[i]);
  c->ctr_bytes = static_cast<size_t>(kNumCtrLines) * 128;
  ChunkParams& p = c->params;
  p.T = L.T;
  p.S = L.S;
  p.variant = d.variant;
  p.SA = d.S;
  p.TA = d.B * d.S;
  p.B = d.B;
  p.NL = d.num_layers;
  p.steps = d.num_steps;
  p.W = d.width;
  p.Hq = d.num_q_heads;
  p.F = d.mlp_dim;
  p.A = d.action_dim;
  p.NN = 2 * d.num_layers + 1;
  p.n_ctx = d.n_ctx;
  p.cap = d.capacity;
  p.mode = d.quant_mode;
  p.scale_bf16 = d.scale_dtype == RFX_DTYPE_BF16;
  p.q_tiles = L.q_tiles;
  p.attn_splits = L.splits;
  p.n_ctx_blocks = L.n_ctx_blocks;
  p.n_blocks = L.n_blocks;
  p.n_attn = L.n_attn;
  p.n_comb = L.n_comb;
  p.n_fin = L.T;
  p.eps = d.eps;
  p.dt = d.dt;
  p.scale_log2 = d.softmax_scale * 1.4426950408889634f;
  for (int i = 0; i < kNumOps; ++i) {
    p.op[i] = L.op[i];
    p.op[i].part = reinterpret_cast<float*>(ws + L.off_part[i]);
  }
  if (d.variant == RFX_CHUNK_PI0) {
    p.state = d.state;
    p.SD = d.state_dim;
    p.w_st = static_cast<const __nv_bfloat16*>(d.w_state);
    p.b_st = static_cast<const __nv_bfloat16*>(d.b_state);
    p.b_atin = d.b_atin;
    p.b_atout = d.b_atout;
    p.temb = static_cast<const __nv_bfloat16*>(d.time_emb);
    p.at_x = reinterpret_cast<__nv_bfloat16*>(ws + L.off_at_x);
    p.at_hid = reinterpret_cast<__nv_bfloat16*>(ws + L.off_at_hid);
    p.st_emb = reinterpret_cast<__nv_bfloat16*>(ws + L.off_st);
    p.new_block = d.new_block;
  }
  p.a1 = d.norm_a1;
  p.a2 = d.mod_a2;
  p.b2 = d.mod_b2;
  p.gate = d.mod_gate;
  p.w_in = static_cast<const __nv_bfloat16*>(d.w_in);
  p.b_in = static_cast<const __nv_bfloat16*>(d.b_in);
  p.w_out = static_cast<const __nv_bfloat16*>(d.w_out);
  p.b_out = static_cast<const __nv_bfloat16*>(d.b_out);
  p.rope = d.rope_table;
  p.rope_max_pos = d.rope_max_pos;
  p.pos = d.positions;
  p.ctx_valid = d.ctx_valid;
  p.x = d.x;
  p.h = reinterpret_cast<__nv_bfloat16*>(ws + L.off_h);
  p.xn = reinterpret_cast<__nv_bfloat16*>(ws + L.off_xn);
  p.q = reinterpret_cast<__nv_bfloat16*>(ws + L.off_q);
  p.kn = reinterpret_cast<__nv_bfloat16*>(ws + L.off_kn);
  p.vn = reinterpret_cast<__nv_bfloat16*>(ws + L.off_vn);
  p.attn_out = reinterpret_cast<__nv_bfloat16*>(ws + L.off_attn);
  p.act = reinterpret_cast<__nv_bfloat16*>(ws + L.off_act);
  p.ws_o = reinterpret_cast<float*>(ws + L.off_ws_o);
  p.ws_ml = reinterpret_cast<float2*>(ws + L.off_ws_ml);
  p.ctr = reinterpret_cast<unsigned*>(ws + L.off_ctr);
  p.status = device_status_ptr();
  p.dbg_h = static_cast<__nv_bfloat16*>(d.debug_hidden);
  p.dbg_attn = static_cast<__nv_bfloat16*>(d.debug_attn);

  // per-layer context pointer tables
  const int NL = d.num_layers;
  std::vector<const void*> ptrs(static_cast<size_t>(6) * NL);
  for (int l = 0; l < NL; ++l) {
    ptrs[0 * NL + l] = d.k_ring[l];
    ptrs[1 * NL + l] = d.v_ring[l];
    ptrs[2 * NL + l] = d.k_scale[l];
    ptrs[3 * NL + l] = d.v_scale[l];
    ptrs[4 * NL + l] = d.quant_mode == RFX_QUANT_U8_REF ? d.k_zp[l] : nullptr;
    ptrs[5 * NL + l] = d.quant_mode == RFX_QUANT_U8_REF ? d.v_zp[l] : nullptr;
  }
  const void** dptr = reinterpret_cast<const void**>(ws + L.off_ptrs);
  p.k_ring = reinterpret_cast<const uint8_t* const*>(dptr);
  p.v_ring = reinterpret_cast<const uint8_t* const*>(dptr + NL);
  p.k_scale = dptr + 2 * NL;
  p.v_scale = dptr + 3 * NL;
  p.k_zp = dptr + 4 * NL;
  p.v_zp = dptr + 5 * NL;
  // task tables
  size_t off = L.off_tasks;
  auto place = [&](size_t bytes) -> char* {
    char* dst = ws + off;
    off += align256(bytes);
    return dst;
  };
  char* st_tasks = place(S.step.size() * sizeof(int4));
  char* in_tasks = place(S.init.size() * sizeof(int4));
  char* st_off = place(S.step_off.size() * sizeof(int));
  char* in_off = place(S.init_off.size() * sizeof(int));
  p.step_tasks = reinterpret_cast<const int4*>(st_tasks);
  p.init_tasks = reinterpret_cast<const int4*>(in_tasks);
  p.step_off = reinterpret_cast<const int*>(st_off);
  p.init_off = reinterpret_cast<const int*>(in_off);
  // synchronous copies: the host vectors die with this call
  rc = check_cuda(cudaMemcpy(dptr, ptrs.data(), ptrs.size() * sizeof(void*), cudaMemcpyHostToDevice), "rfx_chunk: copy");
  if (!rc && !S.step.empty())
    rc = check_cuda(cudaMemcpy(st_tasks, S.step.data(), S.step.size() * sizeof(int4), cudaMemcpyHostToDevice), "copy");
  if (!rc && !S.init.empty())
    rc = check_cuda(cudaMemcpy(in_tasks, S.init.data(), S.init.size() * sizeof(int4), cudaMemcpyHostToDevice), "copy");
  if (!rc) rc = check_cuda(cudaMemcpy(st_off, S.step_off.data(), S.step_off.size() * sizeof(int), cudaMemcpyHostToDevice), "copy");
  if (!rc) rc = check_cuda(cudaMemcpy(in_off, S.init_off.data(), S.init_off.size() * sizeof(int), cudaMemcpyHostToDevice), "copy");

  // tensor maps: weights stacked over layers, activations [T][K], q rows
  const int T = L.T;
  // the action-time MLP's weights are not per layer; its inputs are action-token rows
  const uint64_t wrows[kNumOps] = {static_cast<uint64_t>(NL) * L.op[0].rows, static_cast<uint64_t>(NL) * L.op[1].rows,
                                   static_cast<uint64_t>(NL) * L.op[2].rows, static_cast<uint64_t>(NL) * L.op[3].rows,
                                   static_cast<uint64_t>(L.op[4].rows), static_cast<uint64_t>(L.op[5].rows)};
  const void* wptr[kNumOps] = {d.w_qkv, d.w_o, d.w_gu, d.w_down, d.w_atin, d.w_atout};
  const void* xptr[kNumOps] = {p.xn, p.attn_out, p.xn, p.act, p.at_x, p.at_hid};
  const uint64_t xrows[kNumOps] = {static_cast<uint64_t>(T), static_cast<uint64_t>(T), static_cast<uint64_t>(T),
                                   static_cast<uint64_t>(T), static_cast<uint64_t>(p.TA), static_cast<uint64_t>(p.TA)};
  const int n_ops = d.variant == RFX_CHUNK_PI0 ? kNumOps : kOpDown + 1;
  for (int i = 0; i < n_ops && !rc; ++i) {
    rc = make_tmap_2d(&c->maps.w[i], wptr[i], 2, L.op[i].K, wrows[i], static_cast<uint64_t>(L.op[i].K) * 2, kBK, kBM,
                      true);
    if (!rc)
      rc = make_tmap_2d(&c->maps.x[i], xptr[i], 2, L.op[i].K, xrows[i], static_cast<uint64_t>(L.op[i].K) * 2, kBK,
                        kNT, true);
  }
  if (!rc)
    rc = make_tmap_2d(&c->maps.q, p.q, 2, kD, static_cast<uint64_t>(d.B) * d.num_q_heads * L.S, kD * 2, 64, kQR, true);
  if (!rc) rc = make_tmap_2d(&c->maps.kn, p.kn, 2, kD, static_cast<uint64_t>(T), kD * 2, 64, kKB, true);
  if (!rc) rc = make_tmap_2d(&c->maps.vn, p.vn, 2, kD, static_cast<uint64_t>(T), kD * 2, 64, kKB, true);
  const void* kfn = reinterpret_cast<const void*>(
      chunk_fn(d.variant == RFX_CHUNK_PI0 ? kPi0 : kPi05, d.debug_hidden != nullptr || d.debug_attn != nullptr,
               d.quant_mode == RFX_QUANT_I8_SYM && d.scale_dtype == RFX_DTYPE_F32));
  if (!rc) rc = ensure_smem_attr(kfn, kSmemBytes);
  // the smallest shared-memory carveout that holds the kernel (164 of 228 KB),
  // so the rest of the unified L1 caches local memory and global loads
  if (!rc)
    rc = check_cuda(cudaFuncSetAttribute(kfn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         (kSmemBytes * 100 + 228 * 1024 - 1) / (228 * 1024)),
                    "rfx_chunk: carveout");
  if (!rc) {
    int occ = 0;
    rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kfn, kThreads, kSmemBytes),
                    "rfx_chunk: occupancy");
    if (!rc && occ < 1) rc = set_error(RFX_E_UNSUPPORTED, "rfx_chunk: the kernel does not fit on an SM");
  }
  if (rc) {
    delete c;
    return rc;
  }
  *out = c;
  return RFX_OK;
}

extern "C" int rfx_chunk_run(rfx_chunk* c, void* stream) {
  using namespace rfx;
  if (!c) return set_error(RFX_E_INVAL, "rfx_chunk_run: null chunk");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = check_cuda(cudaMemsetAsync(c->params.ctr, 0, c->ctr_bytes, st), "rfx_chunk_run: clear counters");
  if (rc) return rc;
  // every CTA waits on work of the others: the launch must have all of them
  // resident at once (one per SM), which the cooperative attribute guarantees
  // trace layout: [grid][256 tasks][16] (tasks past 256 of a CTA are not recorded)
  c->params.trace_tasks = 256;
  c->params.dep_limit_ns = dependency_wait_limit_ns();
  c->params.trace = static_cast<unsigned long long*>(trace_buffer(static_cast<size_t>(c->grid) * 256 * 16));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(c->grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // CTA pairs share split-K tiles through DSMEM
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  // without the cooperative attribute (rfx_set_chunk_cooperative(0), for
  // profilers that cannot replay a cooperative launch) only the cluster shape
  // is given
  const bool coop = chunk_cooperative();
  cfg.attrs = coop ? attr : attr + 1;
  cfg.numAttrs = coop ? 2 : 1;
  const ChunkFn fn = chunk_fn(c->params.variant, c->params.dbg_h != nullptr || c->params.dbg_attn != nullptr,
                              c->params.mode == kQuantI8Sym && !c->params.scale_bf16);
  return check_cuda(cudaLaunchKernelEx(&cfg, fn, c->maps, c->params), "rfx_chunk_run: launch");
}

extern "C" int rfx_chunk_destroy(rfx_chunk* c) {
  delete c;
  return RFX_OK;
}

namespace rfx {
int run_chunk_op(rfx_chunk* c, cudaStream_t s) { return rfx_chunk_run(c, s); }
}  // namespace rfx
