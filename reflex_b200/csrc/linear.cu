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
//     accumulates a K-slice in its own TMEM, parks the fp32 partial tile in its
//     shared memory, and after a cluster barrier each CTA reduces a disjoint
//     set of rows over all CTAs' partials through DSMEM in a fixed order
//     (deterministic), then runs the fused epilogue for those rows.
//   * Prologues: TMA load of a bf16 activation, or the RMS/AdaRMS norm
//     computed in-kernel from the residual stream and written to shared memory
//     in the UMMA layout.
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

struct LinParams {
  int T, O, K, S;
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
  int* status;
};

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

// Fused epilogue for rows (i..i+3) and (i+64..i+67) of tile `m` at token t.
template <int EPI>
__device__ __forceinline__ void epilogue4(const LinParams& p, int m, int i, int t, const float (&v0)[4],
                                          const float (&v1)[4]) {
  const int b = t / p.S;
  const long yrow = static_cast<long>(b) * p.y_rps + p.y_off + (t - b * p.S);
  if (EPI == kEpiStore || EPI == kEpiSilu || EPI == kEpiResidual) {
    const int o0 = m * kBM + i, o1 = o0 + 64;
    float r0[4], r1[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a = v0[j], c = v1[j];
      if (EPI != kEpiResidual && p.bias) {
        a += p.bias[o0 + j];
        c += p.bias[o1 + j];
      }
      if (EPI == kEpiSilu) {
        a = silu(bf16_round(a));
        c = silu(bf16_round(c));
      }
      r0[j] = a;
      r1[j] = c;
    }
    __nv_bfloat16* y0 = p.y + yrow * p.ldy + o0;
    __nv_bfloat16* y1 = p.y + yrow * p.ldy + o1;
    if (EPI == kEpiResidual) {
      const float* g = p.gate ? p.gate + static_cast<long>(b) * p.gate_stride : nullptr;
      uint2 old0 = *reinterpret_cast<const uint2*>(y0);
      uint2 old1 = *reinterpret_cast<const uint2*>(y1);
      const __nv_bfloat16* h0 = reinterpret_cast<const __nv_bfloat16*>(&old0);
      const __nv_bfloat16* h1 = reinterpret_cast<const __nv_bfloat16*>(&old1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = bf16_round(r0[j]), c = bf16_round(r1[j]);
        const float ga = g ? bf16_round(__fmul_rn(g[o0 + j], a)) : a;
        const float gc = g ? bf16_round(__fmul_rn(g[o1 + j], c)) : c;
        r0[j] = __fadd_rn(__bfloat162float(h0[j]), ga);
        r1[j] = __fadd_rn(__bfloat162float(h1[j]), gc);
      }
    }
    store_bf16x4(y0, r0);
    store_bf16x4(y1, r1);
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
      int pos = p.pos[t];
      pos = pos < 0 ? 0 : (pos >= p.rope_max_pos ? p.rope_max_pos - 1 : pos);
      const float* cs = p.rope + static_cast<long>(pos) * 256;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x1 = bf16_round(v0[j]);
        const float x2 = bf16_round(v1[j]);
        const float c = cs[d0 + j], sn = cs[128 + d0 + j];
        r0[j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
        r1[j] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
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

template <int NT, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    linear_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const LinParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int XT = NT * 128;  // bytes of one [NT x 64] bf16 activation chunk

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = p.splits > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int m_tile = blockIdx.x / p.splits;
  const int n0 = blockIdx.y * NT;
  const int c_begin = split * p.k_chunks / p.splits;
  const int nch = (split + 1) * p.k_chunks / p.splits - c_begin;
  const int S = p.stages;

  uint8_t* w_ring = smem;
  uint8_t* x_region = smem + S * kWTileBytes;
  float* red = reinterpret_cast<float*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.small_off);
  uint64_t* empty = full + kMaxStages;
  uint64_t* acc_bar = empty + kMaxStages;
  uint64_t* x_ready = acc_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_ready + 1);
  float* rstd_s = reinterpret_cast<float*>(tmem_slot + 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_bar, 1);
    mbar_init(x_ready, 4);
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    if (PRO == kProLoad) tma_prefetch_desc(&tmX);
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
      pdl_wait();
      if (PRO == kProLoad)
        for (int i = 0; i < first; ++i) tma_load_2d(x_region + i * XT, &tmX, &full[i], (c_begin + i) * kBK, n0);
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
    }
  } else {
    const int et = threadIdx.x - 64;  // 0..127
    if (PRO == kProNorm) {
      pdl_wait();
      const int wq = warp - 2;
      for (int tt = wq; tt < NT; tt += 4) {
        const int t = n0 + tt;
        float ss = 0.f;
        if (t < p.T) {
          const __nv_bfloat16* xr = p.x + static_cast<long>(t) * p.ldx;
          for (int k = lane * 8; k < p.K; k += 256) {
            uint4 raw = *reinterpret_cast<const uint4*>(xr + k);
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float2 f = __bfloat1622float2(h2[j]);
              ss = fmaf(f.x, f.x, ss);
              ss = fmaf(f.y, f.y, ss);
            }
          }
          ss = warp_sum(ss);
        }
        if (lane == 0) rstd_s[tt] = t < p.T ? rsqrtf(ss / static_cast<float>(p.K) + p.eps) : 0.f;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int items = nch * NT * 8;
      for (int it = et; it < items; it += 128) {
        const int cc = it & 7;
        const int tt = (it >> 3) % NT;
        const int j = it / (8 * NT);
        const int t = n0 + tt;
        uint4 outv = make_uint4(0u, 0u, 0u, 0u);
        if (t < p.T) {
          const int k = (c_begin + j) * kBK + cc * 8;
          const int b = t / p.S;
          uint4 raw = *reinterpret_cast<const uint4*>(p.x + static_cast<long>(t) * p.ldx + k);
          const __nv_bfloat16* xv = reinterpret_cast<const __nv_bfloat16*>(&raw);
          const float r = rstd_s[tt];
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float v = __fmul_rn(__fmul_rn(__bfloat162float(xv[e]), r), p.a1[k + e]);
            if (p.a2) v = __fmul_rn(v, p.a2[b * p.ab_stride + k + e]);
            if (p.b2) v = __fadd_rn(v, p.b2[b * p.ab_stride + k + e]);
            y[e] = v;
          }
          outv = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                            pack_bf16x2(y[6], y[7]));
        }
        *reinterpret_cast<uint4*>(x_region + j * XT + sw128_offset(tt, cc)) = outv;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(x_ready);
    } else {
      pdl_wait();  // the epilogue reads tensors written by earlier kernels
    }
    // accumulator -> shared partial tile red[t][row]
    const bool ok = mbar_wait(acc_bar, 0, p.status, kDevTimeoutMmaDone);
    tc_fence_after();
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < NT / 16; ++c) {
        uint32_t r[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + c * 16, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) red[(c * 16 + j) * kRedLd + row] = __uint_as_float(r[j]);
      }
    }
    (void)et;
  }
  if (warp == 0) pdl_wait();
  tc_fence_before();
  __syncthreads();
  if (p.splits > 1) cluster_sync();

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
      float v0[4] = {0.f, 0.f, 0.f, 0.f}, v1[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t off0 = red_s + static_cast<uint32_t>((tt * kRedLd + i) * 4);
      const uint32_t off1 = off0 + 64 * 4;
      if (p.splits == 1) {
        const float4 a = *reinterpret_cast<const float4*>(red + tt * kRedLd + i);
        const float4 c = *reinterpret_cast<const float4*>(red + tt * kRedLd + i + 64);
        v0[0] = a.x; v0[1] = a.y; v0[2] = a.z; v0[3] = a.w;
        v1[0] = c.x; v1[1] = c.y; v1[2] = c.z; v1[3] = c.w;
      } else {
        for (int r = 0; r < p.splits; ++r) {
          const float4 a = ld_dsmem_f4(mapa_shared(off0, r));
          const float4 c = ld_dsmem_f4(mapa_shared(off1, r));
          v0[0] += a.x; v0[1] += a.y; v0[2] += a.z; v0[3] += a.w;
          v1[0] += c.x; v1[1] += c.y; v1[2] += c.z; v1[3] += c.w;
        }
      }
      epilogue4<EPI>(p, m_tile, i, t, v0, v1);
    }
  }

  if (p.splits > 1) cluster_sync();
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
}

struct Config {
  int nt, splits, stages, x_slots, small_off, smem;
};

int pick_config(const rfx_linear_desc& d, int num_sms, Config* cfg) {
  int nt = d.n_tile;
  if (nt == 0) nt = d.T <= 64 ? 64 : (d.T <= 128 ? 128 : 256);
  if (nt != 64 && nt != 128 && nt != 256) return set_error(RFX_E_INVAL, "rfx_linear: n_tile must be 64, 128 or 256");
  const int m_tiles = d.O / kBM;
  const int n_tiles = (d.T + nt - 1) / nt;
  const int chunks = d.K / kBK;
  int splits = d.splits;
  if (splits == 0) {
    splits = 1;
    for (int s : {2, 4, 8, 16}) {
      if (s > chunks) break;
      if (m_tiles * n_tiles * s <= num_sms) splits = s;
    }
  }
  if (splits != 1 && splits != 2 && splits != 4 && splits != 8 && splits != 16)
    return set_error(RFX_E_INVAL, "rfx_linear: splits must be 1, 2, 4, 8 or 16");
  if (splits > chunks) return set_error(RFX_E_INVAL, "rfx_linear: splits exceeds K/64");
  const int max_nch = (chunks + splits - 1) / splits;
  const int xt = nt * 128;
  const int small = 2 * kMaxStages * 8 + 16 + 16 + nt * 4 + 64;
  const int budget = kSmemLimit - 1024 - small;
  int stages, x_slots;
  if (d.prologue == RFX_PRO_NORM) {
    x_slots = max_nch;
    const int left = budget - x_slots * xt;
    stages = std::min({max_nch, kMaxStages, left / kWTileBytes});
    if (stages < 1) return set_error(RFX_E_UNSUPPORTED, "rfx_linear: K slice too long for the norm prologue; raise splits");
  } else {
    stages = std::min({max_nch, kMaxStages, budget / (kWTileBytes + xt)});
    x_slots = stages;
    if (stages < 1) return set_error(RFX_E_UNSUPPORTED, "rfx_linear: tile does not fit in shared memory");
  }
  int body = stages * kWTileBytes + x_slots * xt;
  body = std::max(body, nt * kRedLd * 4);
  body = (body + 127) & ~127;
  cfg->nt = nt;
  cfg->splits = splits;
  cfg->stages = stages;
  cfg->x_slots = x_slots;
  cfg->small_off = body;
  cfg->smem = body + small + 1024;
  if (cfg->smem > kSmemLimit) return set_error(RFX_E_UNSUPPORTED, "rfx_linear: shared memory %d too large", cfg->smem);
  return RFX_OK;
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

int validate(const rfx_linear_desc& d) {
  if (d.T < 1 || d.O < kBM || d.O % kBM || d.K < kBK || d.K % kBK || d.tokens_per_batch < 1)
    return set_error(RFX_E_INVAL, "rfx_linear: need T>=1, O%%128==0, K%%64==0, tokens_per_batch>=1 (T=%d O=%d K=%d)",
                     d.T, d.O, d.K);
  if (d.prologue != RFX_PRO_LOAD && d.prologue != RFX_PRO_NORM) return set_error(RFX_E_INVAL, "rfx_linear: prologue");
  if (d.epilogue < RFX_EPI_STORE || d.epilogue > RFX_EPI_GEGLU) return set_error(RFX_E_INVAL, "rfx_linear: epilogue");
  if (!d.w || !d.x || !aligned16(d.w) || !aligned16(d.x) || d.ldx < d.K || d.ldx % 8)
    return set_error(RFX_E_INVAL, "rfx_linear: w/x must be 16-byte aligned and ldx>=K, ldx%%8==0");
  if (d.prologue == RFX_PRO_NORM && !d.norm_a1) return set_error(RFX_E_INVAL, "rfx_linear: norm_a1 required");
  if (d.epilogue == RFX_EPI_QKV_ROPE) {
    if (d.O != (d.num_q_heads + 2) * 256 || !d.q_out || !d.k_out || !d.v_out || !d.rope_table || !d.positions ||
        d.rope_max_pos < 1)
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
  if (d.prologue == RFX_PRO_LOAD)
    rc = make_tmap_2d(tmX, d.x, 2, d.K, d.T, static_cast<uint64_t>(d.ldx) * 2, kBK, cfg.nt, true);
  else
    *tmX = *tmW;  // unused by the norm prologue
  return rc;
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
  const void* fn = select_kernel(cfg.nt, d.prologue, d.epilogue);
  if (!fn) return set_error(RFX_E_INVAL, "rfx_linear: no kernel for this configuration");
  rc = ensure_smem_attr(fn, cfg.smem, cfg.splits > 8);
  if (rc) return rc;
  const int m_tiles = d.O / kBM;
  const int n_tiles = (d.T + cfg.nt - 1) / cfg.nt;
  // an automatically chosen 16-CTA cluster must be co-schedulable; else use 8
  if (d.splits == 0 && cfg.splits == 16 &&
      !cluster_fits(fn, dim3(m_tiles * 16, n_tiles, 1), kThreads, cfg.smem, 16)) {
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
  p.status = device_status_ptr();

  dim3 grid(m_tiles * cfg.splits, n_tiles, 1);
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
