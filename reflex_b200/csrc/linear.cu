// Fused "skinny" linear layers for the action expert: y = epi(pro(x) · Wᵀ)
// with few tokens (T = 50 per stream) and large weights.
//
// B200 design
//   * Swap-AB: the MMA's M dimension is 128 weight rows, N is the token tile
//     (64/128/256), so a 50-token GEMM still runs full-height tcgen05.mma
//     (kind::f16, bf16 in, fp32 accumulate in TMEM).
//   * Weight tiles [128 x 64] bf16 are streamed by TMA (128-byte swizzle) into
//     a ring of shared-memory stages with an L2 evict-first hint; they are
//     issued *before* griddepcontrol.wait, so under programmatic dependent
//     launch the weight stream overlaps the previous kernel's tail.
//   * Split-K across a thread-block cluster: every CTA of the cluster
//     accumulates a K-slice in its own TMEM and parks the fp32 partial tile in
//     its shared memory; after a cluster barrier each CTA reduces a disjoint
//     set of rows over all CTAs' partials through DSMEM in a fixed order
//     (deterministic), with the remote loads batched so their latencies
//     overlap, then runs the fused epilogue for those rows.
//   * Prologues: TMA load of a bf16 activation tile, or the RMS / AdaRMS norm:
//     the raw activation K-slice is TMA-loaded into the UMMA tile, every CTA
//     sums x^2 over its slice, the cluster exchanges the partial sums through
//     DSMEM (the cluster holds the full rows), and the tile is normalized in
//     place in shared memory.
//   * Epilogues work on row pairs (r, r+64) of a tile so RoPE (dims d, d+128)
//     and GELU-tanh(gate)*up see both operands; the weight rows are permuted
//     once at load time (rfx_pack_weight) to put the pairs in one tile.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer, warps 2-5 norm prologue and TMEM readout; all warps reduce.
#include "rfx_internal.h"

#include <algorithm>
#include <mutex>

namespace rfx {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kWTileBytes = kBM * kBK * 2;
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr int kRedLd = 132;  // fp32 row length of the partial tile [t][row] (+4 pad)
constexpr int kSmemLimit = 227 * 1024;

enum { kProLoad = RFX_PRO_LOAD, kProNorm = RFX_PRO_NORM };
enum {
  kEpiStore = RFX_EPI_STORE,
  kEpiSilu = RFX_EPI_SILU,
  kEpiQkvRope = RFX_EPI_QKV_ROPE,
  kEpiResidual = RFX_EPI_RESIDUAL,
  kEpiGeglu = RFX_EPI_GEGLU
};

// Trace events (one 8-byte %globaltimer stamp per event per CTA).
enum {
  kTrStart = 0,
  kTrSetup = 1,
  kTrWIssued = 2,
  kTrPdl = 3,
  kTrFirstFull = 4,
  kTrMmaIssued = 5,
  kTrXFull = 6,
  kTrXReady = 7,
  kTrAcc = 8,
  kTrRed = 9,
  kTrCluster = 10,
  kTrEpi = 11,
  kTrEnd = 12
};

struct LinParams {
  int T, O, K, S;
  int n_tiles;
  int k_chunks;
  int splits;
  int stages;
  int x_slots;
  int small_off;
  const __nv_bfloat16* x;
  int ldx;
  const float* a1;
  const float* a2;
  const float* b2;
  long ab_stride;
  float eps;
  __nv_bfloat16* y;
  int ldy;
  const float* bias;
  const float* gate;
  long gate_stride;
  const float* rope;
  int rope_max_pos;
  const int* pos;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
  int hq;
  int y_rps, y_off;
  int stage_off; // byte offset of the staged epilogue operands (0: fetched in the epilogue)
  int push;      // split-K partials are pushed into the owner CTA's receive buffer
  int recv_off;  // byte offset of the receive buffer [splits][2*pairs][NT] fp32
  int* status;
  unsigned long long* trace;
  // persistent tiles with split-K (ksplit > 1): fp32 partial slots
  // [tile][ksplit][NT][128] and per-tile arrival counters
  int ksplit;
  float* part;
  int* ctr;
  int act;  // activation of the kEpiSilu kernels: 0 SiLU, 1 GELU-tanh (RFX_EPI_GELU)
};

__device__ __forceinline__ void trace(const LinParams& p, int ev) {
  if (kTraceBuilt && p.trace) p.trace[static_cast<long>(blockIdx.x) * 16 + ev] = globaltimer_ns();
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float kBeta = 0.7978845608028654f;  // sqrt(2/pi)
  const float kKappa = 0.044715f;
  const float inner = kBeta * (x + kKappa * x * x * x);
  return 0.5f * x * (1.f + tanhf(inner));
}
__device__ __forceinline__ float silu(float x) { return x / (1.f + expf(-x)); }

__device__ __forceinline__ void store_bf16x4(__nv_bfloat16* p, const float (&v)[4]) {
  uint2 u = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ void unpack_bf16x4(uint2 u, float (&v)[4]) {
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = __bfloat162float(h[j]);
}

// Global operands of one epilogue item, fetched before the reduction so their
// latency overlaps the DSMEM loads.
struct EpiIn {
  float r0[4], r1[4];  // residual (RESIDUAL) or bias (STORE/SILU)
  float g0[4], g1[4];  // gates (RESIDUAL)
  float c[4], s[4];    // RoPE cos / sin (QKV_ROPE)
};

template <int EPI>
__device__ __forceinline__ void epilogue_fetch(const LinParams& p, int m, int i, int t, EpiIn& in) {
  const int b = t / p.S;
  if (EPI == kEpiResidual) {
    const long yrow = static_cast<long>(b) * p.y_rps + p.y_off + (t - b * p.S);
    const int o0 = m * kBM + i;
    unpack_bf16x4(*reinterpret_cast<const uint2*>(p.y + yrow * p.ldy + o0), in.r0);
    unpack_bf16x4(*reinterpret_cast<const uint2*>(p.y + yrow * p.ldy + o0 + 64), in.r1);
    if (p.gate) {
      const float* g = p.gate + static_cast<long>(b) * p.gate_stride + o0;
      const float4 a = *reinterpret_cast<const float4*>(g);
      const float4 c = *reinterpret_cast<const float4*>(g + 64);
      in.g0[0] = a.x; in.g0[1] = a.y; in.g0[2] = a.z; in.g0[3] = a.w;
      in.g1[0] = c.x; in.g1[1] = c.y; in.g1[2] = c.z; in.g1[3] = c.w;
    }
  } else if (EPI == kEpiStore || EPI == kEpiSilu) {
    const int o0 = m * kBM + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      in.r0[j] = p.bias ? p.bias[o0 + j] : 0.f;
      in.r1[j] = p.bias ? p.bias[o0 + 64 + j] : 0.f;
    }
  } else if (EPI == kEpiQkvRope) {
    const int head = m >> 1;
    if (head <= p.hq) {
      int pos = p.pos[t];
      pos = pos < 0 ? 0 : (pos >= p.rope_max_pos ? p.rope_max_pos - 1 : pos);
      const float* cs = p.rope + static_cast<long>(pos) * 256 + (m & 1) * 64 + i;
      const float4 a = *reinterpret_cast<const float4*>(cs);
      const float4 c = *reinterpret_cast<const float4*>(cs + 128);
      in.c[0] = a.x; in.c[1] = a.y; in.c[2] = a.z; in.c[3] = a.w;
      in.s[0] = c.x; in.s[1] = c.y; in.s[2] = c.z; in.s[3] = c.w;
    }
  }
}

// Fused epilogue for rows (i..i+3) and (i+64..i+67) of tile `m` at token t.
template <int EPI>
__device__ __forceinline__ void epilogue_store(const LinParams& p, int m, int i, int t, const float (&v0)[4],
                                               const float (&v1)[4], const EpiIn& in) {
  const int b = t / p.S;
  const long yrow = static_cast<long>(b) * p.y_rps + p.y_off + (t - b * p.S);
  if (EPI == kEpiStore || EPI == kEpiSilu || EPI == kEpiResidual) {
    const int o0 = m * kBM + i;
    float r0[4], r1[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (EPI == kEpiResidual) {
        const float a = bf16_round(p.bias ? v0[j] + p.bias[o0 + j] : v0[j]);
        const float c = bf16_round(p.bias ? v1[j] + p.bias[o0 + 64 + j] : v1[j]);
        const float ga = p.gate ? bf16_round(__fmul_rn(in.g0[j], a)) : a;
        const float gc = p.gate ? bf16_round(__fmul_rn(in.g1[j], c)) : c;
        r0[j] = __fadd_rn(in.r0[j], ga);
        r1[j] = __fadd_rn(in.r1[j], gc);
      } else {
        float a = v0[j] + in.r0[j], c = v1[j] + in.r1[j];
        if (EPI == kEpiSilu) {
          a = p.act ? gelu_tanh(bf16_round(a)) : silu(bf16_round(a));
          c = p.act ? gelu_tanh(bf16_round(c)) : silu(bf16_round(c));
        }
        r0[j] = a;
        r1[j] = c;
      }
    }
    store_bf16x4(p.y + yrow * p.ldy + o0, r0);
    store_bf16x4(p.y + yrow * p.ldy + o0 + 64, r1);
  } else if (EPI == kEpiGeglu) {
    const int f = m * 64 + i;
    float r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float g = bf16_round(v0[j]);
      const float u = bf16_round(v1[j]);
      const float a = bf16_round(gelu_tanh(g));
      r[j] = __fmul_rn(a, u);
    }
    store_bf16x4(p.y + yrow * p.ldy + f, r);
  } else {  // kEpiQkvRope
    const int head = m >> 1;
    const int d0 = (m & 1) * 64 + i;
    const int s = t - b * p.S;
    float r0[4], r1[4];
    if (head <= p.hq) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x1 = bf16_round(v0[j]);
        const float x2 = bf16_round(v1[j]);
        r0[j] = __fsub_rn(__fmul_rn(x1, in.c[j]), __fmul_rn(x2, in.s[j]));
        r1[j] = __fadd_rn(__fmul_rn(x2, in.c[j]), __fmul_rn(x1, in.s[j]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        r0[j] = v0[j];
        r1[j] = v1[j];
      }
    }
    __nv_bfloat16* dst;
    if (head < p.hq)
      dst = p.q_out + ((static_cast<long>(b) * p.hq + head) * p.S + s) * 256;
    else if (head == p.hq)
      dst = p.k_out + static_cast<long>(t) * 256;
    else
      dst = p.v_out + static_cast<long>(t) * 256;
    store_bf16x4(dst + d0, r0);
    store_bf16x4(dst + d0 + 128, r1);
  }
}

// Epilogue operands that do not depend on the accumulator, requested one
// 64-token part ahead by the persistent tile kernel: the residual rows
// (packed bf16) or the RoPE cos / sin of the token.  Gates and bias are
// per-row vectors every item of a thread shares (cache hits), read at store time.
struct EpiPre {
  uint2 y0, y1;
  float4 c, s;
};

template <int EPI>
__device__ __forceinline__ void epilogue_prefetch(const LinParams& p, int m, int i, int t, EpiPre& pre) {
  if (EPI == kEpiResidual) {
    const int b = t / p.S;
    const long yrow = static_cast<long>(b) * p.y_rps + p.y_off + (t - b * p.S);
    const __nv_bfloat16* y = p.y + yrow * p.ldy + m * kBM + i;
    pre.y0 = *reinterpret_cast<const uint2*>(y);
    pre.y1 = *reinterpret_cast<const uint2*>(y + 64);
  } else if (EPI == kEpiQkvRope) {
    if ((m >> 1) <= p.hq) {
      int pos = p.pos[t];
      pos = pos < 0 ? 0 : (pos >= p.rope_max_pos ? p.rope_max_pos - 1 : pos);
      const float* cs = p.rope + static_cast<long>(pos) * 256 + (m & 1) * 64 + i;
      pre.c = *reinterpret_cast<const float4*>(cs);
      pre.s = *reinterpret_cast<const float4*>(cs + 128);
    }
  }
}

// The item's full operand set from its prefetched part (same values as epilogue_fetch).
template <int EPI>
__device__ __forceinline__ void epilogue_expand(const LinParams& p, int m, int i, int t, const EpiPre& pre,
                                                EpiIn& in) {
  if (EPI == kEpiResidual) {
    unpack_bf16x4(pre.y0, in.r0);
    unpack_bf16x4(pre.y1, in.r1);
    if (p.gate) {
      const float* g = p.gate + static_cast<long>(t / p.S) * p.gate_stride + m * kBM + i;
      const float4 a = *reinterpret_cast<const float4*>(g);
      const float4 c = *reinterpret_cast<const float4*>(g + 64);
      in.g0[0] = a.x; in.g0[1] = a.y; in.g0[2] = a.z; in.g0[3] = a.w;
      in.g1[0] = c.x; in.g1[1] = c.y; in.g1[2] = c.z; in.g1[3] = c.w;
    }
  } else if (EPI == kEpiStore || EPI == kEpiSilu) {
    epilogue_fetch<EPI>(p, m, i, t, in);
  } else if (EPI == kEpiQkvRope) {
    in.c[0] = pre.c.x; in.c[1] = pre.c.y; in.c[2] = pre.c.z; in.c[3] = pre.c.w;
    in.s[0] = pre.s.x; in.s[1] = pre.s.y; in.s[2] = pre.s.z; in.s[3] = pre.s.w;
  }
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release_na() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_na() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }

// 128-token tiles run two CTAs per SM: one CTA's epilogue overlaps the
// other's weight / activation stream.
template <int NT, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, NT == 128 ? 2 : 1)
    linear_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const LinParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int XT = NT * 128;  // bytes of one [NT x 64] bf16 activation chunk

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = p.splits > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  // one-dimensional grid: the splits of a tile are consecutive (one cluster),
  // and the token tiles of a weight tile follow each other, so a weight tile
  // is fetched from HBM once and re-read from L2 by its other token tiles
  const int m_tile = blockIdx.x / (p.splits * p.n_tiles);
  const int n0 = (blockIdx.x / p.splits) % p.n_tiles * NT;
  const int c_begin = split * p.k_chunks / p.splits;
  const int nch = (split + 1) * p.k_chunks / p.splits - c_begin;
  const int S = p.stages;
  const bool clustered = p.splits > 1;

  uint8_t* w_ring = smem;
  uint8_t* x_region = smem + S * kWTileBytes;
  float* red = reinterpret_cast<float*>(smem);
  float* recv = reinterpret_cast<float*>(smem + p.recv_off);
  uint8_t* small = smem + p.small_off;
  uint64_t* full = reinterpret_cast<uint64_t*>(small);
  uint64_t* empty = full + kMaxStages;
  uint64_t* acc_bar = reinterpret_cast<uint64_t*>(small + 128);
  uint64_t* x_ready = acc_bar + 1;
  uint64_t* x_full = acc_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(small + 160);
  float* ss_part = reinterpret_cast<float*>(small + 176);
  float* rstd_s = ss_part + NT;
  float* vec_s = rstd_s + NT;  // [3][x_slots*64]: a1, a2, b2 of this CTA's K-slice

  if (threadIdx.x == 0) trace(p, kTrStart);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_bar, 1);
    mbar_init(x_ready, 4);
    mbar_init(x_full, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, NT);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  if (threadIdx.x == 0) trace(p, kTrSetup);
  // the norm prologue exchanges partial sums over the cluster; the producer and
  // MMA warps take part in that barrier phase without waiting for it here
  if (PRO == kProNorm && clustered && warp < 2) cluster_arrive_relaxed();

  int issued = 0;  // chunks whose TMA the producer issued
  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t bytes = kWTileBytes + (PRO == kProLoad ? XT : 0);
      const int first = nch < S ? nch : S;
      for (int i = 0; i < first; ++i) {
        mbar_arrive_expect_tx(&full[i], bytes);
        tma_load_2d_hint(w_ring + i * kWTileBytes, &tmW, &full[i], (c_begin + i) * kBK, m_tile * kBM, pol);
      }
      trace(p, kTrWIssued);
      pdl_wait();
      trace(p, kTrPdl);
      if (PRO == kProLoad) {
        for (int i = 0; i < first; ++i) tma_load_2d(x_region + i * XT, &tmX, &full[i], (c_begin + i) * kBK, n0);
      } else {
        mbar_arrive_expect_tx(x_full, nch * XT);
        for (int j = 0; j < nch; ++j) tma_load_2d(x_region + j * XT, &tmX, x_full, (c_begin + j) * kBK, n0);
      }
      issued = first;
      for (int i = first; i < nch; ++i) {
        const int s = i % S;
        if (!mbar_wait(&empty[s], ((i / S) - 1) & 1, p.status, kDevTimeoutStageEmpty)) break;
        mbar_arrive_expect_tx(&full[s], bytes);
        tma_load_2d_hint(w_ring + s * kWTileBytes, &tmW, &full[s], (c_begin + i) * kBK, m_tile * kBM, pol);
        if (PRO == kProLoad) tma_load_2d(x_region + s * XT, &tmX, &full[s], (c_begin + i) * kBK, n0);
        issued = i + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(kBM, NT, true);
      bool ok = true;
      if (PRO == kProNorm) ok = mbar_wait(x_ready, 0, p.status, kDevTimeoutXReady);
      for (int i = 0; i < nch && ok; ++i) {
        const int s = i % S;
        if (!mbar_wait(&full[s], (i / S) & 1, p.status, kDevTimeoutTmaFull)) break;
        if (i == 0) trace(p, kTrFirstFull);
        tc_fence_after();
        const uint32_t a_base = smem_u32(w_ring + s * kWTileBytes);
        const uint32_t b_base = smem_u32(x_region + (PRO == kProLoad ? s : i) * XT);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t ad = make_sdesc_sw128(a_base + kk * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(b_base + kk * 32, 16, 1024);
          umma_f16_ss(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(acc_bar);
      trace(p, kTrMmaIssued);
    }
  } else {
    const int et = threadIdx.x - 64;  // 0..127
    const int wq = warp - 2;
    pdl_wait();
    if (p.stage_off > 0) {
      // while the weights stream, fetch the epilogue's global operands of every
      // item of this CTA into shared memory (4 items' loads in flight per thread)
      const int pairs = 64 / p.splits;
      const int quads = pairs / 4;
      const int items = quads * NT;
      EpiIn* stage = reinterpret_cast<EpiIn*>(smem + p.stage_off);
      for (int it0 = et; it0 < items; it0 += 4 * 128) {
        EpiIn in[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int it = it0 + u * 128;
          const int t = n0 + it / quads;
          if (it < items && t < p.T) epilogue_fetch<EPI>(p, m_tile, split * pairs + (it % quads) * 4, t, in[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (it0 + u * 128 < items) stage[it0 + u * 128] = in[u];
      }
    }
    if (PRO == kProNorm) {
      // norm vectors of this CTA's K-slice -> shared memory
      const int kw4 = nch * kBK / 4;  // float4s per vector (<= 256)
      const bool shared_vec = p.ab_stride == 0;
      {
        float4 va[2], vb[2], vc[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int e = et + q * 128;
          if (e < kw4) {
            const int k = c_begin * kBK + 4 * e;
            va[q] = *reinterpret_cast<const float4*>(p.a1 + k);
            vb[q] = (shared_vec && p.a2) ? *reinterpret_cast<const float4*>(p.a2 + k) : make_float4(1.f, 1.f, 1.f, 1.f);
            vc[q] = (shared_vec && p.b2) ? *reinterpret_cast<const float4*>(p.b2 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int e = et + q * 128;
          if (e < kw4) {
            reinterpret_cast<float4*>(vec_s)[e] = va[q];
            reinterpret_cast<float4*>(vec_s + p.x_slots * kBK)[e] = vb[q];
            reinterpret_cast<float4*>(vec_s + 2 * p.x_slots * kBK)[e] = vc[q];
          }
        }
      }
      const bool ok = mbar_wait(x_full, 0, p.status, kDevTimeoutTmaFull);
      if (et == 0) trace(p, kTrXFull);
      // partial sum of squares of every token over this CTA's K-slice
      for (int tt = wq; tt < NT; tt += 4) {
        float ss = 0.f;
        if (ok) {
          for (int c = lane; c < nch * 8; c += 32) {
            const uint4 raw = *reinterpret_cast<const uint4*>(x_region + (c >> 3) * XT + sw128_offset(tt, c & 7));
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __bfloat1622float2(h2[j]);
              ss = fmaf(f.x, f.x, ss);
              ss = fmaf(f.y, f.y, ss);
            }
          }
        }
        ss = warp_sum(ss);
        if (lane == 0) ss_part[tt] = ss;
      }
      if (clustered) {
        cluster_arrive_release_na();
        cluster_wait_na();
      } else {
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      // rstd from the partial sums of every CTA in the cluster (fixed order)
      for (int tt = et; tt < NT; tt += 128) {
        float tot = 0.f;
        if (clustered) {
          float part[16];
          const uint32_t a = smem_u32(ss_part + tt);
#pragma unroll
          for (int r = 0; r < 16; ++r)
            if (r < p.splits) part[r] = ld_dsmem_f32(mapa_shared(a, r));
#pragma unroll
          for (int r = 0; r < 16; ++r)
            if (r < p.splits) tot += part[r];
        } else {
          tot = ss_part[tt];
        }
        rstd_s[tt] = rsqrtf(tot / static_cast<float>(p.K) + p.eps);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      // normalize the tile in place
      const int items = nch * NT * 8;
      for (int it = et; it < items; it += 128) {
        const int cc = it & 7;
        const int tt = (it >> 3) % NT;
        const int j = it / (8 * NT);
        const int t = n0 + tt;
        uint4* cell = reinterpret_cast<uint4*>(x_region + j * XT + sw128_offset(tt, cc));
        uint4 outv = make_uint4(0u, 0u, 0u, 0u);
        if (t < p.T) {
          const uint4 raw = *cell;
          const __nv_bfloat16* xv = reinterpret_cast<const __nv_bfloat16*>(&raw);
          const float r = rstd_s[tt];
          const int e0 = j * kBK + cc * 8;
          const long bo = static_cast<long>(t / p.S) * p.ab_stride + c_begin * kBK + e0;
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float a1 = vec_s[e0 + e];
            const float a2 = shared_vec ? vec_s[p.x_slots * kBK + e0 + e] : (p.a2 ? p.a2[bo + e] : 1.f);
            const float b2 = shared_vec ? vec_s[2 * p.x_slots * kBK + e0 + e] : (p.b2 ? p.b2[bo + e] : 0.f);
            float v = __fmul_rn(__fmul_rn(__bfloat162float(xv[e]), r), a1);
            if (p.a2) v = __fmul_rn(v, a2);
            if (p.b2) v = __fadd_rn(v, b2);
            y[e] = v;
          }
          outv = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                            pack_bf16x2(y[6], y[7]));
        }
        *cell = outv;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(x_ready);
      if (et == 0) trace(p, kTrXReady);
    }
    // accumulator -> shared partial tile red[t][row]
    const bool ok = mbar_wait(acc_bar, 0, p.status, kDevTimeoutMmaDone);
    tc_fence_after();
    if (et == 0) trace(p, kTrAcc);
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    if (ok) {
      // push mode: this row's partial goes to the CTA that reduces its pair
      const int pairs = 64 / p.splits;
      const int pr = row & 63;
      const int owner = pr / pairs;
      const int lr = (pr - owner * pairs) + (row >= 64 ? pairs : 0);
      const uint32_t dst =
          p.push ? mapa_shared(smem_u32(recv + static_cast<long>(split * 2 * pairs + lr) * NT), owner) : 0u;
#pragma unroll
      for (int c0 = 0; c0 < NT / 16; c0 += 4) {
        uint32_t r[4][16];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (c0 + q < NT / 16) tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + (c0 + q) * 16, r[q]);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (c0 + q >= NT / 16) continue;
          if (p.push) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              st_dsmem_f4(dst + static_cast<uint32_t>(((c0 + q) * 16 + 4 * j) * 4), __uint_as_float(r[q][4 * j]),
                          __uint_as_float(r[q][4 * j + 1]), __uint_as_float(r[q][4 * j + 2]),
                          __uint_as_float(r[q][4 * j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) red[((c0 + q) * 16 + j) * kRedLd + row] = __uint_as_float(r[q][j]);
          }
        }
      }
    }
    if (et == 0) trace(p, kTrRed);
  }
  pdl_wait();
  tc_fence_before();
  __syncthreads();
  if (clustered) {
    if (PRO == kProNorm && warp < 2) cluster_wait_na();  // completes the prologue phase
    cluster_sync();
  }
  if (threadIdx.x == 64) trace(p, kTrCluster);

  // ---- reduction over the cluster + fused epilogue (all threads) ----
  {
    const int pairs = 64 / p.splits;
    const int quads = pairs / 4;
    const int pair0 = split * pairs;
    const int items = quads * NT;
    const uint32_t red_s = smem_u32(red);
    for (int it = threadIdx.x; it < items; it += kThreads) {
      const int qd = it % quads;
      const int tt = it / quads;
      const int t = n0 + tt;
      if (t >= p.T) continue;
      const int i = pair0 + qd * 4;
      EpiIn in;
      if (p.stage_off > 0)
        in = reinterpret_cast<const EpiIn*>(smem + p.stage_off)[it];
      else
        epilogue_fetch<EPI>(p, m_tile, i, t, in);
      float v0[4] = {0.f, 0.f, 0.f, 0.f}, v1[4] = {0.f, 0.f, 0.f, 0.f};
      if (p.push) {
        // every CTA of the cluster pushed its partial of these rows here: local sums, fixed order
        const int lr0 = qd * 4;
        for (int src = 0; src < p.splits; ++src) {
          const float* base = recv + static_cast<long>(src * 2 * pairs) * NT + tt;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            v0[j] += base[(lr0 + j) * NT];
            v1[j] += base[(pairs + lr0 + j) * NT];
          }
        }
      } else if (!clustered) {
        const float4 a = *reinterpret_cast<const float4*>(red + tt * kRedLd + i);
        const float4 c = *reinterpret_cast<const float4*>(red + tt * kRedLd + i + 64);
        v0[0] = a.x; v0[1] = a.y; v0[2] = a.z; v0[3] = a.w;
        v1[0] = c.x; v1[1] = c.y; v1[2] = c.z; v1[3] = c.w;
      } else {
        const uint32_t off0 = red_s + static_cast<uint32_t>((tt * kRedLd + i) * 4);
        const uint32_t off1 = off0 + 64 * 4;
        for (int r0 = 0; r0 < p.splits; r0 += 8) {
          float4 a[8], c[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (r0 + q < p.splits) {
              a[q] = ld_dsmem_f4(mapa_shared(off0, r0 + q));
              c[q] = ld_dsmem_f4(mapa_shared(off1, r0 + q));
            }
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (r0 + q < p.splits) {
              v0[0] += a[q].x; v0[1] += a[q].y; v0[2] += a[q].z; v0[3] += a[q].w;
              v1[0] += c[q].x; v1[1] += c[q].y; v1[2] += c[q].z; v1[3] += c[q].w;
            }
          }
        }
      }
      epilogue_store<EPI>(p, m_tile, i, t, v0, v1, in);
    }
  }
  if (threadIdx.x == 64) trace(p, kTrEpi);

  // pull mode reads peers' shared memory: keep it alive until every CTA is done
  if (clustered && !p.push) cluster_sync();
  // drain: a producer that stopped early waits (bounded) for its TMA writes
  if (warp == 0 && lane == 0) {
    for (int i = (issued > S ? issued - S : 0); i < issued; ++i) {
      const int s = i % S;
      mbar_wait(&full[s], (i / S) & 1, p.status, kDevTimeoutTmaFull);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, NT);
  }
  if (threadIdx.x == 0) trace(p, kTrEnd);
}

// ----------------------------------------------------- persistent tiles ---
// Many tokens (T > 128, load prologue): one CTA per SM walks work units
// u = blockIdx.x, blockIdx.x + gridDim.x, ... in weight-tile-major order (a
// weight tile's token tiles are adjacent, so they run at the same time and
// the tile comes from HBM once); a unit is a tile, or one of its K splits
// when split-K is on.  The producer streams W / X k-steps through a 4-stage
// ring without stopping at unit boundaries; the MMA issuer fills two TMEM
// accumulators alternately; warps 2-9 drain the other one (TMEM ->
// shared-memory transpose -> the fused epilogue, four items per thread with
// their operands in flight together), so a tile's epilogue runs under the
// next unit's mainloop.
// Layout per token tile NT (128 or 256): a 4-stage ring of W [128 x 64] +
// X [NT x 64] bf16, the epilogue's transpose buffer for 64 tokens at a time.
constexpr int kPStages = 4;
constexpr int kTThreads = 320;  // TMA producer warp, MMA warp, 8 epilogue warps
template <int NT>
struct TilesLayout {
  static constexpr int kStage = kWTileBytes + NT * 128;
  static constexpr int kOffRed = kPStages * kStage;            // [64 tokens][kRedLd] fp32
  static constexpr int kOffSmall = kOffRed + 64 * kRedLd * 4;
  static constexpr int kSmem = kOffSmall + 128 + 1024;
};
static_assert(TilesLayout<256>::kSmem <= kSmemLimit, "256-token tiles fit in shared memory");
// TMEM columns of the two accumulators (allocations are powers of two)
template <int NT>
constexpr uint32_t tiles_tmem_cols() {
  return NT <= 128 ? 256u : 512u;
}

template <int NT, int EPI>
__global__ void __launch_bounds__(kTThreads, 1)
    linear_tiles_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                        const LinParams p) {
  using Lay = TilesLayout<NT>;
  constexpr int kPStage = Lay::kStage;
  constexpr int kPOffRed = Lay::kOffRed;
  constexpr int kPOffSmall = Lay::kOffSmall;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* red = reinterpret_cast<float*>(smem + kPOffRed);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPOffSmall);
  uint64_t* empty = full + kPStages;
  uint64_t* acc_full = empty + kPStages;  // [2]
  uint64_t* acc_free = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_free + 2);
  // work units: (tile, K split), the splits of a tile adjacent
  const int n_units = (p.O / kBM) * p.n_tiles * p.ksplit;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_free[i], kTThreads / 32 - 2);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tiles_tmem_cols<NT>());
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  if (threadIdx.x == 0) trace(p, kTrSetup);
  int issued = 0;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      bool ok = true;
      bool waited = false;
      for (int un = blockIdx.x; un < n_units && ok; un += gridDim.x) {
        const int tile = un / p.ksplit, ks = un % p.ksplit;
        const int m = tile / p.n_tiles, n0 = (tile % p.n_tiles) * NT;
        const int kc0 = ks * p.k_chunks / p.ksplit, kc1 = (ks + 1) * p.k_chunks / p.ksplit;
        for (int kc = kc0; kc < kc1; ++kc) {
          const int s = issued % kPStages;
          if (issued >= kPStages &&
              !(ok = mbar_wait(&empty[s], ((issued / kPStages) - 1) & 1, p.status, kDevTimeoutStageEmpty)))
            break;
          uint8_t* st = smem + s * kPStage;
          mbar_arrive_expect_tx(&full[s], kPStage);
          tma_load_2d_hint(st, &tmW, &full[s], kc * kBK, m * kBM, pol);
          if (!waited) {  // the activations come from the previous kernel
            pdl_wait();
            waited = true;
          }
          tma_load_2d(st + kWTileBytes, &tmX, &full[s], kc * kBK, n0);
          ++issued;
        }
      }
      if (!waited) pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(kBM, NT, true);
      const uint64_t a0 = make_sdesc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t b0 = make_sdesc_sw128(smem_u32(smem + kWTileBytes), 16, 1024);
      bool ok = true;
      int it = 0, tl = 0;
      for (int un = blockIdx.x; un < n_units && ok; un += gridDim.x, ++tl) {
        const int ks = un % p.ksplit;
        const int kc0 = ks * p.k_chunks / p.ksplit, kc1 = (ks + 1) * p.k_chunks / p.ksplit;
        const int buf = tl & 1;
        if (tl >= 2 && !(ok = mbar_wait(&acc_free[buf], ((tl >> 1) - 1) & 1, p.status, kDevTimeoutMmaDone))) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * NT;
        for (int kc = kc0; kc < kc1; ++kc, ++it) {
          const int s = it % kPStages;
          if (!(ok = mbar_wait(&full[s], (it / kPStages) & 1, p.status, kDevTimeoutTmaFull))) break;
          tc_fence_after();
          const uint64_t off = static_cast<uint64_t>((s * kPStage) >> 4);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16_ss(acc, a0 + off + kk * 2, b0 + off + kk * 2, idesc, (kc > kc0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
    }
  } else {
    pdl_wait();
    // 8 epilogue warps, two per TMEM lane quadrant: warps 2-5 take the first
    // 32 token columns of each 64-token part, warps 6-9 the other 32
    const int et = threadIdx.x - 64;  // 0..255
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int ch = et >> 7;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    int tl = 0;
    int* last_s = reinterpret_cast<int*>(acc_free + 2) + 1;  // the split counter outcome for all workers
    for (int un = blockIdx.x; un < n_units; un += gridDim.x, ++tl) {
      const int tile = un / p.ksplit, ks = un % p.ksplit;
      const int m = tile / p.n_tiles, n0 = (tile % p.n_tiles) * NT;
      const int buf = tl & 1;
      // a thread's items: one row group, tokens 16 apart; the first part's
      // operands are requested before the accumulator is waited for
      const int irow = (et & 15) * 4;
      EpiPre cur[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = n0 + (et >> 4) + 16 * u;
        if (t < p.T) epilogue_prefetch<EPI>(p, m, irow, t, cur[u]);
      }
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&acc_full[buf], (tl >> 1) & 1, p.status, kDevTimeoutMmaDone);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      // every epilogue warp agrees before anyone leaves the loop
      uint32_t all;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, 256, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(all)
          : "r"(ok ? 1u : 0u)
          : "memory");
      if (!all) break;
      tc_fence_after();
      const uint32_t acc = tmem + buf * NT + lane_base;
      bool split_last = false;
      if (p.ksplit > 1) {
        // this split's fp32 partial [t][row] to its slot, then the tile's arrival
        // counter; the last split to arrive sums every slot in split order
        float* slot = p.part + (static_cast<long>(tile) * p.ksplit + ks) * NT * 128;
#pragma unroll 1
        for (int h = 0; h < NT / 64; ++h) {
          uint32_t r[2][16];
#pragma unroll
          for (int c = 0; c < 2; ++c) tmem_ld16(acc + 64 * h + 32 * ch + 16 * c, r[c]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 16; ++e)
              __stcg(slot + (64 * h + 32 * ch + 16 * c + e) * 128 + row, __uint_as_float(r[c][e]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_free[buf]);
        __threadfence();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (et == 0) {
          const int old = atomicAdd(p.ctr + tile, 1);
          if (old == p.ksplit - 1) {
            __threadfence();
            p.ctr[tile] = 0;  // ready for the next launch
          }
          *last_s = old == p.ksplit - 1 ? 1 : 0;
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        split_last = *last_s != 0;
        if (!split_last) continue;
        __threadfence();
      }
      // parts of 64 token columns: accumulator row `row` -> red[t][row], then
      // the fused epilogue of those tokens
#pragma unroll 1
      for (int h = 0; h < NT / 64; ++h) {
        if (split_last) {
          // the sum of the splits' partials of tokens 64h .. 64h+63 in split
          // order: per split 32 KB contiguous, float4 k * 256 + et holding
          // token 8k + et / 32, rows 4 (et % 32) .. +3
          const float4* base =
              reinterpret_cast<const float4*>(p.part + static_cast<long>(tile) * p.ksplit * NT * 128 + (64 * h) * 128);
          float4 sum[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) sum[j] = __ldcg(base + j * 256 + et);
#pragma unroll 1
          for (int q = 1; q < p.ksplit; ++q) {
            const float4* src = base + static_cast<long>(q) * (NT * 128 / 4);
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __ldcg(src + j * 256 + et);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              sum[j].x += v[j].x;
              sum[j].y += v[j].y;
              sum[j].z += v[j].z;
              sum[j].w += v[j].w;
            }
          }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(red + (8 * j + (et >> 5)) * kRedLd + 4 * lane) = sum[j];
        } else {
          uint32_t r[2][16];
#pragma unroll
          for (int c = 0; c < 2; ++c) tmem_ld16(acc + 64 * h + 32 * ch + 16 * c, r[c]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 16; ++e) red[(32 * ch + 16 * c + e) * kRedLd + row] = __uint_as_float(r[c][e]);
          if (h == NT / 64 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_free[buf]);
          }
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        // items: 16 groups of 4 row pairs x 64 tokens; 16 consecutive threads
        // cover one token's 64 pairs (coalesced stores); the next part's
        // operands are requested before this part's stores
        const int t0 = n0 + 64 * h;
        EpiPre nxt[4];
        if (h + 1 < NT / 64) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int t = t0 + 64 + (et >> 4) + 16 * u;
            if (t < p.T) epilogue_prefetch<EPI>(p, m, irow, t, nxt[u]);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int tt = (et >> 4) + 16 * u;
          if (t0 + tt >= p.T) continue;
          EpiIn in;
          epilogue_expand<EPI>(p, m, irow, t0 + tt, cur[u], in);
          const float4 a = *reinterpret_cast<const float4*>(red + tt * kRedLd + irow);
          const float4 c = *reinterpret_cast<const float4*>(red + tt * kRedLd + irow + 64);
          const float v0[4] = {a.x, a.y, a.z, a.w};
          const float v1[4] = {c.x, c.y, c.z, c.w};
          epilogue_store<EPI>(p, m, irow, t0 + tt, v0, v1, in);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) cur[u] = nxt[u];
        asm volatile("bar.sync 1, 256;" ::: "memory");  // red is free again
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // drain: a producer that stopped early waits (bounded) for its TMA writes
  if (warp == 0 && lane == 0)
    for (int i = (issued > kPStages ? issued - kPStages : 0); i < issued; ++i)
      mbar_wait(&full[i % kPStages], (i / kPStages) & 1, p.status, kDevTimeoutTmaFull);
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tiles_tmem_cols<NT>());
  }
  if (threadIdx.x == 0) trace(p, kTrEnd);
}

struct Config {
  int nt, splits, stages, x_slots, small_off, smem, push, recv_off, stage_off;
};

int small_bytes(int nt, bool norm, int x_slots) {
  const int b = 176 + 8 * nt + (norm ? 3 * x_slots * kBK * 4 : 0);
  return (b + 127) & ~127;
}

int pick_config(const rfx_linear_desc& d, int num_sms, Config* cfg) {
  int nt = d.n_tile;
  if (nt == 0) nt = d.T <= 64 ? 64 : 128;
  if (nt != 64 && nt != 128 && nt != 256) return set_error(RFX_E_INVAL, "rfx_linear: n_tile must be 64, 128 or 256");
  // 128-token tiles: two CTAs per SM (each within half of the SM's shared memory)
  const int per_sm = nt == 128 ? 2 : 1;
  const int smem_limit = nt == 128 ? 113 * 1024 : kSmemLimit;
  const bool norm = d.prologue == RFX_PRO_NORM;
  const int m_tiles = d.O / kBM;
  const int n_tiles = (d.T + nt - 1) / nt;
  const int chunks = d.K / kBK;
  int splits = d.splits;
  if (splits == 0) {
    splits = 1;
    // clusters of at most 8 CTAs: larger ones wait for whole free GPCs, which
    // kernels overlapping under programmatic dependent launch rarely leave
    for (int s : {2, 4, 8}) {
      if (s > chunks) break;
      if (m_tiles * n_tiles * s <= num_sms * per_sm) splits = s;
    }
  }
  if (splits != 1 && splits != 2 && splits != 4 && splits != 8)
    return set_error(RFX_E_INVAL, "rfx_linear: splits must be 1, 2, 4 or 8");
  if (splits > chunks) return set_error(RFX_E_INVAL, "rfx_linear: splits exceeds K/64");
  const int xt = nt * 128;
  auto budget_for = [&](int xs) { return smem_limit - 1024 - small_bytes(nt, norm, xs); };
  if (norm && d.splits == 0) {
    // the normalized K-slice of a CTA stays resident: split K further (or
    // shrink the token tile) until it fits next to one weight stage
    auto fits = [&](int s) {
      const int xs = (chunks + s - 1) / s;
      return xs * xt <= budget_for(xs) - kWTileBytes;
    };
    while (!fits(splits) && splits < 8 && splits * 2 <= chunks) splits *= 2;
    if (!fits(splits) && d.n_tile == 0 && nt > 64) {
      rfx_linear_desc smaller = d;
      smaller.n_tile = nt / 2;
      return pick_config(smaller, num_sms, cfg);
    }
  }
  const int max_nch = (chunks + splits - 1) / splits;
  // Preferred layout: split-K partials pushed into a dedicated receive buffer
  // and the epilogue operands staged in shared memory (TMA-fed X only).  When
  // that does not fit next to one pipeline stage, keep the push and fetch the
  // operands in the epilogue (pulling partials over DSMEM costs a remote
  // round trip per split and item: 19.0 against 17.0 us for a 400-token
  // o_proj), then pull.
  const int items = (16 / splits) * nt;
  const int want_push = (!norm && splits > 1) ? 1 : 0;
  int want_stage = (!norm && d.epilogue != RFX_EPI_GEGLU) ? items * static_cast<int>(sizeof(EpiIn)) : 0;
  if (want_stage > 48 * 1024) want_stage = 0;
  const int options[4][2] = {{want_push, want_stage}, {want_push, 0}, {0, want_stage}, {0, 0}};
  for (const auto& opt : options) {
    const int push = opt[0], stage_bytes = opt[1];
    const int recv_bytes = push ? 128 * nt * 4 : 0;
    int stages, x_slots;
    if (norm) {
      x_slots = max_nch;
      const int left = budget_for(x_slots) - x_slots * xt;
      stages = std::min({max_nch, kMaxStages, left / kWTileBytes});
      if (stages < 1)
        return set_error(RFX_E_UNSUPPORTED, "rfx_linear: K slice too long for the norm prologue; raise splits");
    } else {
      stages = std::min({max_nch, kMaxStages, (budget_for(0) - recv_bytes - stage_bytes) / (kWTileBytes + xt)});
      x_slots = stages;
      if (stages < 1) continue;
    }
    int body = stages * kWTileBytes + x_slots * xt;
    if (!push) body = std::max(body, nt * kRedLd * 4);
    body = (body + 127) & ~127;
    const int smem = body + recv_bytes + stage_bytes + small_bytes(nt, norm, x_slots) + 1024;
    if (smem > smem_limit) continue;
    cfg->nt = nt;
    cfg->splits = splits;
    cfg->stages = stages;
    cfg->x_slots = x_slots;
    cfg->push = push;
    cfg->recv_off = body;
    cfg->stage_off = stage_bytes ? body + recv_bytes : 0;
    cfg->small_off = body + recv_bytes + stage_bytes;
    cfg->smem = smem;
    return RFX_OK;
  }
  return set_error(RFX_E_UNSUPPORTED, "rfx_linear: tile does not fit in shared memory (n_tile %d)", nt);
}

template <int NT, int PRO, int EPI>
const void* kernel_ptr() {
  return reinterpret_cast<const void*>(linear_kernel<NT, PRO, EPI>);
}

template <int NT, int PRO>
const void* select_epi(int epi) {
  switch (epi) {
    case kEpiStore: return kernel_ptr<NT, PRO, kEpiStore>();
    case kEpiSilu: return kernel_ptr<NT, PRO, kEpiSilu>();
    case kEpiQkvRope: return kernel_ptr<NT, PRO, kEpiQkvRope>();
    case kEpiResidual: return kernel_ptr<NT, PRO, kEpiResidual>();
    case kEpiGeglu: return kernel_ptr<NT, PRO, kEpiGeglu>();
  }
  return nullptr;
}
template <int NT>
const void* select_pro(int pro, int epi) {
  return pro == kProNorm ? select_epi<NT, kProNorm>(epi) : select_epi<NT, kProLoad>(epi);
}
const void* select_kernel(int nt, int pro, int epi) {
  switch (nt) {
    case 64: return select_pro<64>(pro, epi);
    case 128: return select_pro<128>(pro, epi);
    case 256: return select_pro<256>(pro, epi);
  }
  return nullptr;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// RFX_EPI_GELU runs the SiLU epilogue's kernels with the activation switched
int kernel_epi(int epi) { return epi == RFX_EPI_GELU ? RFX_EPI_SILU : epi; }

int validate(const rfx_linear_desc& d) {
  if (d.T < 1 || d.O < kBM || d.O % kBM || d.K < kBK || d.K % kBK || d.tokens_per_batch < 1)
    return set_error(RFX_E_INVAL, "rfx_linear: need T>=1, O%%128==0, K%%64==0, tokens_per_batch>=1 (T=%d O=%d K=%d)",
                     d.T, d.O, d.K);
  if (d.prologue != RFX_PRO_LOAD && d.prologue != RFX_PRO_NORM) return set_error(RFX_E_INVAL, "rfx_linear: prologue");
  if (d.epilogue < RFX_EPI_STORE || d.epilogue > RFX_EPI_GELU) return set_error(RFX_E_INVAL, "rfx_linear: epilogue");
  if (!d.w || !d.x || !aligned16(d.w) || !aligned16(d.x) || d.ldx < d.K || d.ldx % 8)
    return set_error(RFX_E_INVAL, "rfx_linear: w/x must be 16-byte aligned and ldx>=K, ldx%%8==0");
  if (d.prologue == RFX_PRO_NORM &&
      (!d.norm_a1 || !aligned16(d.norm_a1) || (d.norm_a2 && !aligned16(d.norm_a2)) ||
       (d.norm_b2 && !aligned16(d.norm_b2)) || d.norm_ab_stride % 4))
    return set_error(RFX_E_INVAL, "rfx_linear: norm vectors must be 16-byte aligned (norm_a1 required)");
  if (d.gate && (reinterpret_cast<uintptr_t>(d.gate) & 15u || d.gate_stride % 4))
    return set_error(RFX_E_INVAL, "rfx_linear: gate must be 16-byte aligned with gate_stride%%4==0");
  if (d.epilogue == RFX_EPI_QKV_ROPE) {
    if (d.O != (d.num_q_heads + 2) * 256 || !d.q_out || !d.k_out || !d.v_out || !d.rope_table || !d.positions ||
        d.rope_max_pos < 1 || !aligned16(d.rope_table))
      return set_error(RFX_E_INVAL, "rfx_linear: QKV_ROPE needs O=(Hq+2)*256 and q/k/v/rope/positions");
  } else if (d.epilogue == RFX_EPI_GEGLU) {
    if (!d.y || d.ldy < d.O / 2 || d.ldy % 4) return set_error(RFX_E_INVAL, "rfx_linear: GEGLU output");
  } else {
    if (!d.y || d.ldy < d.O || d.ldy % 4) return set_error(RFX_E_INVAL, "rfx_linear: output y/ldy");
  }
  if (d.y_rows_per_batch > 0 && (d.y_row_offset < 0 || d.y_row_offset + d.tokens_per_batch > d.y_rows_per_batch))
    return set_error(RFX_E_INVAL, "rfx_linear: y_row_offset + tokens_per_batch must fit y_rows_per_batch");
  return RFX_OK;
}

}  // namespace

namespace {
// K splits of the persistent kernel's tiles: the count (1..4) that finishes
// the units soonest, waves of units x their length (1 / ksplit) plus a tenth
// of a unit for the partials' round trip.  A split keeps at least 8 k-steps,
// and at least 32 when it adds a round of units: a short split unit costs
// about as much as a long one (its partial store, the sum and the epilogue
// dominate), so it pays only where it fills idle SMs in the same round (a
// 400-token o_proj, K = 2048, as 4 x 8 k-steps: 15.8 us against 17.1 us for
// the per-tile kernel's in-cluster split; the same rule at 1600 tokens would
// have tripled the rounds).  The partial slots stay within 64 MB.
constexpr int kSplitMaxTiles = 16384;  // tiles the fixed counter block serves
int pick_ksplit(int tiles, int k_chunks, int nt, int nsm) {
  int best = 1;
  double best_t = static_cast<double>((tiles + nsm - 1) / nsm);
  if (tiles > kSplitMaxTiles) return 1;
  const int rounds1 = (tiles + nsm - 1) / nsm;
  for (int s = 2; s <= 4; ++s) {
    if (k_chunks / s < 8 || static_cast<size_t>(tiles) * s * nt * 128 * 4 > (size_t(64) << 20)) break;
    if (tiles * s > rounds1 * nsm && k_chunks / s < 32) continue;
    const double t = static_cast<double>((tiles * s + nsm - 1) / nsm) / s + 0.1;
    if (t < best_t - 1e-9) {
      best_t = t;
      best = s;
    }
  }
  return best;
}

// Split-K workspace of the persistent kernel: a fixed 64 KB of per-tile
// arrival counters (int) then fp32 partial slots [tile][ksplit][nt][128].
// The counter block has the same place and size for every shape, so GEMMs of
// different shapes can take turns on one workspace: no launch's partials ever
// land on another shape's counters (each launch leaves its counters zero).
size_t split_ctr_bytes(int) { return static_cast<size_t>(kSplitMaxTiles) * 4; }
size_t split_workspace_bytes(int tiles, int ksplit, int nt) {
  if (ksplit <= 1) return 0;
  return split_ctr_bytes(tiles) + static_cast<size_t>(tiles) * ksplit * nt * 128 * 4;
}

// Many tokens (T > 128) with the load prologue and automatic tiling go to the
// persistent tile kernel with 128-, 192- or 256-token tiles: the width with
// the least (rounds of tiles over the SMs) x (width + 300), a round's time
// growing with the width on top of a fixed part of about 300 tokens' worth
// (set-up, pipeline fill, the last epilogue; fitted to measured times of the
// frame and 64-stream shapes).  With 128-token tiles, K is split over several CTAs when
// the tiles alone leave SMs idle and the caller gave a workspace
// (`assume_ws`: as if it had).  Without a split and with fewer than half an
// SM's worth of 128-token tiles, the per-tile kernel's in-cluster split-K
// keeps more SMs busy: nt = 0.
struct TilesPlan {
  int nt = 0, ksplit = 1;
  size_t ws = 0;
};
TilesPlan plan_tiles(const rfx_linear_desc& d, int nsm, bool assume_ws) {
  TilesPlan t;
  if (d.prologue != RFX_PRO_LOAD || d.splits != 0 || d.n_tile != 0 || d.T <= 128) return t;
  const int m_tiles = d.O / kBM;
  long best = -1;
  for (int nt : {128, 192, 256}) {
    const int tiles = m_tiles * ((d.T + nt - 1) / nt);
    const long c = static_cast<long>((tiles + nsm - 1) / nsm) * (nt + 300);
    if (best < 0 || c < best) {
      t.nt = nt;
      best = c;
    }
  }
  if (t.nt != 128) return t;
  const int tiles = m_tiles * ((d.T + t.nt - 1) / t.nt);
  t.ksplit = pick_ksplit(tiles, d.K / kBK, t.nt, nsm);
  t.ws = split_workspace_bytes(tiles, t.ksplit, t.nt);
  const bool have_ws =
      assume_ws || (d.workspace && d.workspace_bytes >= t.ws && (reinterpret_cast<uintptr_t>(d.workspace) & 255) == 0);
  if (t.ksplit > 1 && !have_ws) {
    t.ksplit = 1;
    t.ws = 0;
  }
  if (t.ksplit == 1 && 2 * tiles < nsm) t.nt = 0;
  return t;
}

template <int NT, int EPI>
const void* tiles_ptr() {
  return reinterpret_cast<const void*>(linear_tiles_kernel<NT, EPI>);
}
template <int NT>
const void* select_tiles_nt(int epi) {
  switch (epi) {
    case kEpiStore: return tiles_ptr<NT, kEpiStore>();
    case kEpiSilu: return tiles_ptr<NT, kEpiSilu>();
    case kEpiQkvRope: return tiles_ptr<NT, kEpiQkvRope>();
    case kEpiResidual: return tiles_ptr<NT, kEpiResidual>();
    case kEpiGeglu: return tiles_ptr<NT, kEpiGeglu>();
  }
  return nullptr;
}
const void* select_tiles(int nt, int epi) {
  return nt == 256 ? select_tiles_nt<256>(epi) : nt == 192 ? select_tiles_nt<192>(epi) : select_tiles_nt<128>(epi);
}
int tiles_smem(int nt) {
  return nt == 256 ? TilesLayout<256>::kSmem : nt == 192 ? TilesLayout<192>::kSmem : TilesLayout<128>::kSmem;
}

LinParams lin_params(const rfx_linear_desc& d) {
  LinParams p{};
  p.T = d.T;
  p.O = d.O;
  p.K = d.K;
  p.S = d.tokens_per_batch;
  p.k_chunks = d.K / kBK;
  p.x = static_cast<const __nv_bfloat16*>(d.x);
  p.ldx = d.ldx;
  p.a1 = d.norm_a1;
  p.a2 = d.norm_a2;
  p.b2 = d.norm_b2;
  p.ab_stride = d.norm_ab_stride;
  p.eps = d.eps;
  p.y = static_cast<__nv_bfloat16*>(d.y);
  p.ldy = d.ldy;
  p.bias = d.bias;
  p.gate = d.gate;
  p.gate_stride = d.gate_stride;
  p.rope = d.rope_table;
  p.rope_max_pos = d.rope_max_pos;
  p.pos = d.positions;
  p.q_out = static_cast<__nv_bfloat16*>(d.q_out);
  p.k_out = static_cast<__nv_bfloat16*>(d.k_out);
  p.v_out = static_cast<__nv_bfloat16*>(d.v_out);
  p.hq = d.num_q_heads;
  p.y_rps = d.y_rows_per_batch > 0 ? d.y_rows_per_batch : d.tokens_per_batch;
  p.y_off = d.y_rows_per_batch > 0 ? d.y_row_offset : 0;
  p.status = device_status_ptr();
  p.act = d.epilogue == RFX_EPI_GELU ? 1 : 0;
  return p;
}

int launch_linear_tiles(const rfx_linear_desc& d, const CUtensorMap* tmW, const CUtensorMap* tmX, const TilesPlan& tp,
                        int nsm, cudaStream_t stream, bool pdl) {
  const int nt = tp.nt;
  const void* fn = select_tiles(nt, kernel_epi(d.epilogue));
  if (!fn) return set_error(RFX_E_INVAL, "rfx_linear: no tile kernel for this epilogue");
  const int smem = tiles_smem(nt);
  int rc = ensure_smem_attr(fn, smem);
  if (rc) return rc;
  LinParams p = lin_params(d);
  p.splits = 1;
  p.n_tiles = (d.T + nt - 1) / nt;
  const int tiles = (d.O / kBM) * p.n_tiles;
  p.ksplit = tp.ksplit;
  if (p.ksplit > 1) {
    p.ctr = static_cast<int*>(d.workspace);
    p.part = reinterpret_cast<float*>(static_cast<uint8_t*>(d.workspace) + split_ctr_bytes(tiles));
  }
  const int grid = std::min(tiles * p.ksplit, nsm);
  p.trace = static_cast<unsigned long long*>(trace_buffer(static_cast<size_t>(grid) * 16));
  CUtensorMap w = *tmW, x = *tmX;
  return launch_kernel(fn, dim3(grid), dim3(kTThreads), static_cast<size_t>(smem), stream, pdl, 1, w, x, p);
}
}  // namespace

int build_linear_maps(const rfx_linear_desc& d, CUtensorMap* tmW, CUtensorMap* tmX) {
  int rc = validate(d);
  if (rc) return rc;
  int nsm = 148;
  rfx_num_sms(&nsm);
  Config cfg;
  rc = pick_config(d, nsm, &cfg);
  if (rc) return rc;
  rc = make_tmap_2d(tmW, d.w, 2, d.K, d.O, static_cast<uint64_t>(d.K) * 2, kBK, kBM, true);
  if (rc) return rc;
  const int pnt = plan_tiles(d, nsm, false).nt;
  return make_tmap_2d(tmX, d.x, 2, d.K, d.T, static_cast<uint64_t>(d.ldx) * 2, kBK, pnt ? pnt : cfg.nt, true);
}

int launch_linear(const rfx_linear_desc& d, const CUtensorMap* tmW, const CUtensorMap* tmX, cudaStream_t stream,
                  bool pdl) {
  int rc = validate(d);
  if (rc) return rc;
  int nsm = 148;
  rfx_num_sms(&nsm);
  Config cfg;
  rc = pick_config(d, nsm, &cfg);
  if (rc) return rc;
  const TilesPlan tp = plan_tiles(d, nsm, false);
  if (tp.nt) return launch_linear_tiles(d, tmW, tmX, tp, nsm, stream, pdl);
  const void* fn = select_kernel(cfg.nt, d.prologue, kernel_epi(d.epilogue));
  if (!fn) return set_error(RFX_E_INVAL, "rfx_linear: no kernel for this configuration");
  rc = ensure_smem_attr(fn, cfg.smem, cfg.splits > 8);
  if (rc) return rc;
  const int m_tiles = d.O / kBM;
  const int n_tiles = (d.T + cfg.nt - 1) / cfg.nt;
  // an automatically chosen 16-CTA cluster must be co-schedulable; else use 8
  if (d.splits == 0 && cfg.splits == 16 &&
      !cluster_fits(fn, dim3(m_tiles * 16 * n_tiles, 1, 1), kThreads, cfg.smem, 16)) {
    rfx_linear_desc d8 = d;
    d8.splits = 8;
    rc = pick_config(d8, nsm, &cfg);
    if (rc) return rc;
    rc = ensure_smem_attr(fn, cfg.smem, false);
    if (rc) return rc;
  }

  LinParams p{};
  p.T = d.T;
  p.O = d.O;
  p.K = d.K;
  p.S = d.tokens_per_batch;
  p.k_chunks = d.K / kBK;
  p.splits = cfg.splits;
  p.stages = cfg.stages;
  p.x_slots = cfg.x_slots;
  p.small_off = cfg.small_off;
  p.x = static_cast<const __nv_bfloat16*>(d.x);
  p.ldx = d.ldx;
  p.a1 = d.norm_a1;
  p.a2 = d.norm_a2;
  p.b2 = d.norm_b2;
  p.ab_stride = d.norm_ab_stride;
  p.eps = d.eps;
  p.y = static_cast<__nv_bfloat16*>(d.y);
  p.ldy = d.ldy;
  p.bias = d.bias;
  p.gate = d.gate;
  p.gate_stride = d.gate_stride;
  p.rope = d.rope_table;
  p.rope_max_pos = d.rope_max_pos;
  p.pos = d.positions;
  p.q_out = static_cast<__nv_bfloat16*>(d.q_out);
  p.k_out = static_cast<__nv_bfloat16*>(d.k_out);
  p.v_out = static_cast<__nv_bfloat16*>(d.v_out);
  p.hq = d.num_q_heads;
  p.y_rps = d.y_rows_per_batch > 0 ? d.y_rows_per_batch : d.tokens_per_batch;
  p.y_off = d.y_rows_per_batch > 0 ? d.y_row_offset : 0;
  p.push = cfg.push;
  p.recv_off = cfg.recv_off;
  p.stage_off = cfg.stage_off;
  p.status = device_status_ptr();
  p.act = d.epilogue == RFX_EPI_GELU ? 1 : 0;
  p.trace = static_cast<unsigned long long*>(trace_buffer(m_tiles * cfg.splits * n_tiles * 16));

  p.n_tiles = n_tiles;
  dim3 grid(m_tiles * cfg.splits * n_tiles, 1, 1);
  CUtensorMap w = *tmW, x = *tmX;
  return launch_kernel(fn, grid, dim3(kThreads), static_cast<size_t>(cfg.smem), stream, pdl, cfg.splits, w, x, p);
}

// ------------------------------------------------------------ packing ---
namespace {
__global__ void pack_rows_kernel(const __nv_bfloat16* __restrict__ src, __nv_bfloat16* __restrict__ dst, int kind,
                                 int rows, int K) {
  const int r = blockIdx.x;
  const int m = r / kBM, rr = r % kBM;
  int srow;
  if (kind == RFX_PACK_QKV_ROPE) {
    const int head = m >> 1, half = m & 1;
    srow = head * 256 + (rr < 64 ? half * 64 + rr : 128 + half * 64 + (rr - 64));
  } else {
    const int f = rows / 2;
    srow = rr < 64 ? m * 64 + rr : f + m * 64 + (rr - 64);
  }
  const uint4* s = reinterpret_cast<const uint4*>(src + static_cast<long>(srow) * K);
  uint4* d = reinterpret_cast<uint4*>(dst + static_cast<long>(r) * K);
  for (int i = threadIdx.x; i < K / 8; i += blockDim.x) d[i] = s[i];
}
}  // namespace

}  // namespace rfx

extern "C" int rfx_pack_weight(int kind, const void* src, void* dst, int rows, int K, void* stream) {
  using namespace rfx;
  if (!src || !dst || src == dst) return set_error(RFX_E_INVAL, "rfx_pack_weight: src/dst");
  if (K % 8 || (reinterpret_cast<uintptr_t>(src) & 15u) || (reinterpret_cast<uintptr_t>(dst) & 15u))
    return set_error(RFX_E_INVAL, "rfx_pack_weight: K%%8 and 16-byte alignment required");
  if (kind == RFX_PACK_QKV_ROPE) {
    if (rows % 256) return set_error(RFX_E_INVAL, "rfx_pack_weight: QKV rows must be a multiple of 256");
  } else if (kind == RFX_PACK_GATE_UP) {
    if (rows % 128) return set_error(RFX_E_INVAL, "rfx_pack_weight: gate/up rows must be a multiple of 128");
  } else {
    return set_error(RFX_E_INVAL, "rfx_pack_weight: kind");
  }
  pack_rows_kernel<<<rows, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(src), static_cast<__nv_bfloat16*>(dst), kind, rows, K);
  return check_cuda(cudaGetLastError(), "rfx_pack_weight");
}

extern "C" int rfx_linear(const rfx_linear_desc* desc, void* stream) {
  using namespace rfx;
  if (!desc) return set_error(RFX_E_INVAL, "rfx_linear: null descriptor");
  CUtensorMap w, x;
  int rc = build_linear_maps(*desc, &w, &x);
  if (rc) return rc;
  return launch_linear(*desc, &w, &x, static_cast<cudaStream_t>(stream), pdl_enabled());
}

extern "C" int rfx_linear_workspace_size(const rfx_linear_desc* desc, size_t* bytes) {
  using namespace rfx;
  if (!desc || !bytes) return set_error(RFX_E_INVAL, "rfx_linear_workspace_size: null argument");
  *bytes = 0;
  int rc = validate(*desc);
  if (rc) return rc;
  int nsm = 148;
  rfx_num_sms(&nsm);
  *bytes = plan_tiles(*desc, nsm, true).ws;
  return RFX_OK;
}
