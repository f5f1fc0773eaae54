// Partitioned attention of the new (suffix) tokens over a quantized context
// ring plus the new tokens' own bf16 K/V, on tcgen05 tensor cores.
//
// Work decomposition
//   rows  = num_q_heads x S query rows of one stream, stacked head-major (MQA:
//           every head shares the single KV head, so heads become MMA rows);
//           tiles of 128 rows (MMA M = 128).
//   keys  = ceil(n_ctx/64) context blocks of 64 ring slots, then ceil(S/64)
//           blocks of new keys.  Grid (q_tiles, kv_splits, B); split sp owns
//           a contiguous range of key blocks and runs an online softmax over
//           them; with kv_splits > 1 the partial (O, m, l) go to a workspace
//           and a combine kernel merges them (log-sum-exp weights).
//
// Per key block (64 keys):
//   TMA  : int8/uint8 K and V rows [64 x 256] -> shared staging
//   conv : int8 -> bf16 K tile (exact; per-token scale applied to the fp32
//          scores) and int8 -> f16 V tile (exact; per-token scale folded into
//          the probabilities), or, for the reference uint8 scheme, the
//          reference's dequantize ((q - zp) * scale, rounded per op to the
//          scale dtype) -> bf16 K / f16 V.  New keys are copied from bf16.
//   MMA1 : S[128 x 64] = Q[128 x 256] · Kᵀ  (bf16, fp32 in TMEM)
//   soft : tcgen05.ld rows, mask, online max / sum, P = p * v_scale -> f16
//          shared tile (conditional rescale of O in TMEM when the running max
//          grows by more than 2^8)
//   MMA2 : O[128 x 256] += P[128 x 64] · V[64 x 256]  (f16, V MN-major)
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer, warps 2-5 convert / softmax / epilogue (warp w reads TMEM lanes
// 32*(w%4) .. +31, i.e. one query row per thread).
#include "rfx_internal.h"

#include <algorithm>
#include <mutex>
#include <unordered_map>

namespace rfx {
namespace {

constexpr int kD = 256;
constexpr int kKB = 64;
constexpr int kQR = 128;
constexpr int kThreads = 192;

// shared memory map (offsets from a 1024-aligned base)
constexpr int kOffQ = 0;                     // 4 x [128 x 64] bf16, 64 KB
constexpr int kOffK = kOffQ + 4 * 16384;     // 4 x [64 x 64] bf16, 32 KB
constexpr int kOffV = kOffK + 4 * 8192;      // 4 x [64 x 64] f16 (MN-major blocks), 32 KB
constexpr int kOffP = kOffV + 4 * 8192;      // [128 x 64] f16, 16 KB
constexpr int kOffSK = kOffP + 16384;        // int8 K staging [64 x 256], 16 KB
constexpr int kOffSV = kOffSK + 16384;       // int8 V staging, 16 KB
constexpr int kOffScale = kOffSV + 16384;    // ks, vs, kdq, vdq, kzp, vzp (fp32), nb (int32): 7 x 64
constexpr int kOffBar = kOffScale + 8 * 64 * 4;
constexpr int kSmemBytes = kOffBar + 256 + 1024;

struct AttnParams {
  int B, Hq, S, cap, n_ctx, mode, scale_bf16;
  int q_tiles, splits, n_ctx_blocks, n_blocks;
  const __nv_bfloat16* k_new;
  const __nv_bfloat16* v_new;
  const void* k_scale;
  const void* v_scale;
  const void* k_zp;
  const void* v_zp;
  const unsigned char* ctx_valid;
  const int* new_block;
  float scale_log2;
  __nv_bfloat16* out;
  float* ws_o;
  float2* ws_ml;
  int* status;
  unsigned long long* trace;
  // dense key source (RFX_KV_DENSE): [B][Lk] per-key score scale (log2
  // units), value scale and mask add (0 or -inf), bf16 K / f16 V [B][Lk][D]
  float* key_ks;
  float* key_vs;
  float* key_add;
  int* key_nb;  // block id of the key (-1 for context keys; new_block[k] for new key k)
  __nv_bfloat16* kd;
  __half* vd;
  int Lk;
};

// Trace events (one %globaltimer stamp per event per CTA, see rfx_set_trace).
enum {
  kTrStart = 0, kTrSetup = 1, kTrIssued = 2, kTrKv = 3, kTrConv = 4, kTrS = 5, kTrP = 6, kTrO = 7, kTrEnd = 8,
  kTrSLoaded = 9, kTrMax = 10, kTrExp = 11, kTrOLoaded = 12, kTrOStored = 13
};

__device__ __forceinline__ void trace(const AttnParams& p, int ev) {
  if (kTraceBuilt && p.trace)
    p.trace[((static_cast<long>(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * 16 + ev] =
        globaltimer_ns();
}

__device__ __forceinline__ float load_scalar(const void* p, long i, bool bf16) {
  return bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]) : static_cast<const float*>(p)[i];
}
__device__ __forceinline__ float round_to(float x, bool bf16) { return bf16 ? bf16_round(x) : x; }

// Converts 16 consecutive quantized values of one key row into bf16 (K) or
// f16 (V) and stores them as two 16-byte chunks of a 128-byte-swizzled tile.
template <bool IS_K>
__device__ __forceinline__ void convert16(const uint8_t* src, uint8_t* tile_base, int key, int g, int mode,
                                          bool sbf16, float sc, float zp) {
  uint4 raw = *reinterpret_cast<const uint4*>(src);
  const uint8_t* b8 = reinterpret_cast<const uint8_t*>(&raw);
  float f[16];
  if (mode == kQuantI8Sym) {
#pragma unroll
    for (int e = 0; e < 16; ++e) f[e] = static_cast<float>(static_cast<int8_t>(b8[e]));
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float t = round_to(__fsub_rn(static_cast<float>(b8[e]), zp), sbf16);
      f[e] = round_to(__fmul_rn(t, sc), sbf16);
    }
  }
  uint32_t w[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) w[e] = IS_K ? pack_bf16x2(f[2 * e], f[2 * e + 1]) : pack_f16x2(f[2 * e], f[2 * e + 1]);
  uint8_t* atom = tile_base + (g >> 2) * 8192;
  const int c0 = (g & 3) * 2;
  *reinterpret_cast<uint4*>(atom + sw128_offset(key, c0)) = make_uint4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<uint4*>(atom + sw128_offset(key, c0 + 1)) = make_uint4(w[4], w[5], w[6], w[7]);
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
  const int blk_begin = sp * p.n_blocks / p.splits;
  const int blk_end = (sp + 1) * p.n_blocks / p.splits;
  const int nbl = blk_end - blk_begin;

  uint8_t* sQ = smem + kOffQ;
  uint8_t* sK = smem + kOffK;
  uint8_t* sV = smem + kOffV;
  uint8_t* sP = smem + kOffP;
  uint8_t* stK = smem + kOffSK;
  uint8_t* stV = smem + kOffSV;
  float* ks_s = reinterpret_cast<float*>(smem + kOffScale);
  float* vs_s = ks_s + 64;
  float* kdq_s = vs_s + 64;  // reference-scheme dequant scales and zero points
  float* vdq_s = kdq_s + 64;
  float* kzp_s = vdq_s + 64;
  float* vzp_s = kzp_s + 64;
  int* nb_s = reinterpret_cast<int*>(vzp_s + 64);  // block ids of the new keys of the block
  float* kadd_s = reinterpret_cast<float*>(nb_s + 64);  // 0 or -inf (masked key)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;
  uint64_t* stage_free = bars + 2;
  uint64_t* conv_done = bars + 3;
  uint64_t* s_full = bars + 4;
  uint64_t* p_ready = bars + 5;
  uint64_t* o_full = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);

  if (threadIdx.x == 0) trace(p, kTrStart);
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(kv_full, 1);
    mbar_init(stage_free, 4);
    mbar_init(conv_done, 4);
    mbar_init(s_full, 1);
    mbar_init(p_ready, 4);
    mbar_init(o_full, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmO = tmem, tmS = tmem + 256;
  pdl_launch_dependents();
  if (threadIdx.x == 0) trace(p, kTrSetup);

  // The quantized context (ring payload, scales, validity) is not written
  // while a chunk runs, so its first block is fetched and converted before
  // griddepcontrol.wait, overlapping the kernel that produces Q.  Everything
  // that reads the new tokens' Q/K/V waits first.
  const long q_row0 = static_cast<long>(b) * p.Hq * p.S + static_cast<long>(qt) * kQR;
  int issued_ctx = 0;

  if (warp == 0) {
    if (lane == 0 && nbl > 0) {
      auto issue_kv = [&](int j) {
        mbar_arrive_expect_tx(kv_full, 2 * 16384);
        const int row = b * p.cap + j * kKB;
        tma_load_2d(stK, &tmK, kv_full, 0, row);
        tma_load_2d(stV, &tmV, kv_full, 0, row);
        ++issued_ctx;
      };
      if (blk_begin < p.n_ctx_blocks) issue_kv(blk_begin);
      pdl_wait();
      mbar_arrive_expect_tx(q_full, 4 * 16384);
      for (int a = 0; a < 4; ++a) tma_load_2d(sQ + a * 16384, &tmQ, q_full, a * 64, static_cast<int>(q_row0));
      for (int jl = 1; jl < nbl; ++jl) {
        const int j = blk_begin + jl;
        if (j >= p.n_ctx_blocks) break;
        if (!mbar_wait(stage_free, (issued_ctx - 1) & 1, p.status, kDevTimeoutStageEmpty)) break;
        issue_kv(j);
      }
      trace(p, kTrIssued);
    }
    pdl_wait();
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0 && nbl > 0) {
      constexpr uint32_t idesc_s = make_idesc_f16(kQR, kKB, true);
      constexpr uint32_t idesc_o = make_idesc_f16(kQR, kD, false, true);
      bool ok = mbar_wait(q_full, 0, p.status, kDevTimeoutTmaFull);
      for (int jl = 0; jl < nbl && ok; ++jl) {
        if (!(ok = mbar_wait(conv_done, jl & 1, p.status, kDevTimeoutConvert))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const int a = ks >> 2, kk = ks & 3;
          const uint64_t ad = make_sdesc_sw128(smem_u32(sQ + a * 16384) + kk * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(smem_u32(sK + a * 8192) + kk * 32, 16, 1024);
          umma_f16_ss(tmS, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        if (!(ok = mbar_wait(p_ready, jl & 1, p.status, kDevTimeoutConvert))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kKB / 16; ++ks) {
          const uint64_t ad = make_sdesc_sw128(smem_u32(sP) + ks * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(smem_u32(sV) + ks * 2048, 8192, 1024);
          umma_f16_ss(tmO, ad, bd, idesc_o, (jl > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(o_full);
      }
    }
  } else {
    const int et = threadIdx.x - 64;  // 0..127
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row inside the tile == TMEM lane
    const int R = qt * kQR + r;      // stacked row inside the stream
    const bool row_valid = R < p.Hq * p.S;
    const int s_row = row_valid ? R % p.S : 0;
    const int h_row = row_valid ? R / p.S : 0;
    const int my_block = (row_valid && p.new_block) ? p.new_block[s_row] : 0;
    const bool sbf16 = p.scale_bf16 != 0;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    int ctx_iter = 0;
    bool ok = true;
    bool waited = false;  // griddepcontrol.wait done by this thread

    for (int jl = 0; jl < nbl && ok; ++jl) {
      const int j = blk_begin + jl;
      const bool is_ctx = j < p.n_ctx_blocks;
      if (jl > 0) ok = mbar_wait(o_full, (jl - 1) & 1, p.status, kDevTimeoutMmaDone);
      if (!ok) break;
      if (!is_ctx && !waited) {
        pdl_wait();
        waited = true;
      }
      // ---- convert block j into sK / sV ----
      if (is_ctx) {
        if (et < 64) {
          const long slot = static_cast<long>(j) * kKB + et;
          const long gi = static_cast<long>(b) * p.cap + (slot < p.cap ? slot : p.cap - 1);
          bool valid = slot < p.n_ctx;
          if (valid && p.ctx_valid) valid = p.ctx_valid[gi] != 0;
          // score (log2 units) = acc * ks + kadd; kadd = -inf masks the key
          kadd_s[et] = valid ? 0.f : -INFINITY;
          if (p.mode == kQuantI8Sym) {
            ks_s[et] = valid ? static_cast<const float*>(p.k_scale)[gi] * p.scale_log2 : 0.f;
            vs_s[et] = valid ? static_cast<const float*>(p.v_scale)[gi] : 0.f;
          } else {
            ks_s[et] = valid ? p.scale_log2 : 0.f;
            vs_s[et] = 1.f;
            kdq_s[et] = load_scalar(p.k_scale, gi, sbf16);
            vdq_s[et] = load_scalar(p.v_scale, gi, sbf16);
            kzp_s[et] = load_scalar(p.k_zp, gi, sbf16);
            vzp_s[et] = load_scalar(p.v_zp, gi, sbf16);
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (!(ok = mbar_wait(kv_full, ctx_iter & 1, p.status, kDevTimeoutTmaFull))) break;
        ++ctx_iter;
        if (et == 0) trace(p, kTrKv);
        for (int it = et; it < 2 * kKB * 16; it += 128) {
          const bool isv = it >= kKB * 16;
          const int w = isv ? it - kKB * 16 : it;
          const int key = w >> 4, g = w & 15;
          float sc = 0.f, zp = 0.f;
          if (p.mode != kQuantI8Sym) {
            sc = isv ? vdq_s[key] : kdq_s[key];
            zp = isv ? vzp_s[key] : kzp_s[key];
          }
          if (isv)
            convert16<false>(stV + key * kD + g * 16, sV, key, g, p.mode, sbf16, sc, zp);
          else
            convert16<true>(stK + key * kD + g * 16, sK, key, g, p.mode, sbf16, sc, zp);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(stage_free);
      } else {
        const int nb0 = (j - p.n_ctx_blocks) * kKB;
        if (et < 64) {
          const int kk = nb0 + et;
          ks_s[et] = kk < p.S ? p.scale_log2 : 0.f;  // block-causal visibility is applied per row
          kadd_s[et] = kk < p.S ? 0.f : -INFINITY;
          vs_s[et] = 1.f;
          nb_s[et] = (kk < p.S && p.new_block) ? p.new_block[kk] : 0;
        }
        for (int it = et; it < 2 * kKB * 32; it += 128) {
          const bool isv = it >= kKB * 32;
          const int w = isv ? it - kKB * 32 : it;
          const int key = w >> 5, c = w & 31;  // 32 chunks of 8 elements per key
          const int kk = nb0 + key;
          uint4 raw = make_uint4(0u, 0u, 0u, 0u);
          if (kk < p.S) {
            const __nv_bfloat16* src = (isv ? p.v_new : p.k_new) + (static_cast<long>(b) * p.S + kk) * kD + c * 8;
            raw = *reinterpret_cast<const uint4*>(src);
          }
          uint8_t* atom = (isv ? sV : sK) + (c >> 3) * 8192;
          if (isv) {
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
            uint32_t w4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float2 f = __bfloat1622float2(h2[e]);
              w4[e] = pack_f16x2(f.x, f.y);
            }
            raw = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
          *reinterpret_cast<uint4*>(atom + sw128_offset(key, c & 7)) = raw;
        }
      }
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (lane == 0) mbar_arrive(conv_done);
      if (et == 0) trace(p, kTrConv);
      if (!waited) {
        pdl_wait();
        waited = true;
      }

      // ---- softmax on S ----
      if (!(ok = mbar_wait(s_full, jl & 1, p.status, kDevTimeoutMmaDone))) break;
      tc_fence_after();
      if (et == 0) trace(p, kTrS);
      float z[kKB];
      {
        uint32_t rr[kKB / 16][16];
#pragma unroll
        for (int c = 0; c < kKB / 16; ++c) tmem_ld16(tmS + lane_base + c * 16, rr[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < kKB / 16; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) z[c * 16 + e] = __uint_as_float(rr[c][e]);
      }
      if (et == 0) trace(p, kTrSLoaded);
      // scores in log2 units: one FMA per key from float4 vectors, masked keys
      // become -inf; the max is a 4-way tree so the chain is short
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      const bool causal = !is_ctx && p.new_block != nullptr;
#pragma unroll
      for (int c = 0; c < kKB / 4; ++c) {
        const float4 km = reinterpret_cast<const float4*>(ks_s)[c];
        const float4 ka = reinterpret_cast<const float4*>(kadd_s)[c];
        z[4 * c + 0] = fmaf(z[4 * c + 0], km.x, ka.x);
        z[4 * c + 1] = fmaf(z[4 * c + 1], km.y, ka.y);
        z[4 * c + 2] = fmaf(z[4 * c + 2], km.z, ka.z);
        z[4 * c + 3] = fmaf(z[4 * c + 3], km.w, ka.w);
        if (causal) {
          const int4 nb = reinterpret_cast<const int4*>(nb_s)[c];
          if (nb.x > my_block) z[4 * c + 0] = -INFINITY;
          if (nb.y > my_block) z[4 * c + 1] = -INFINITY;
          if (nb.z > my_block) z[4 * c + 2] = -INFINITY;
          if (nb.w > my_block) z[4 * c + 3] = -INFINITY;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) mx[e] = fmaxf(mx[e], z[4 * c + e]);
      }
      const float bmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      float m_new = fmaxf(m_run, bmax);
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
      if (et == 0) trace(p, kTrMax);
      // p = 2^(z - m): ex2 of -inf is +0, so masked keys need no branch
      const float m_sub = m_use == -INFINITY ? 0.f : m_use;
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
      float pv[kKB];
#pragma unroll
      for (int c = 0; c < kKB / 4; ++c) {
        const float4 vsc = reinterpret_cast<const float4*>(vs_s)[c];
        const float vv[4] = {vsc.x, vsc.y, vsc.z, vsc.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float pe = ex2_approx(z[4 * c + e] - m_sub);
          ps[e] += pe;
          pv[4 * c + e] = pe * vv[e];
        }
      }
      const float psum = (ps[0] + ps[1]) + (ps[2] + ps[3]);
      l_run = l_run * alpha + psum;
      if (et == 0) trace(p, kTrExp);
      m_run = m_use;
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c0 = 0; c0 < kD / 16; c0 += 4) {
          uint32_t rr[4][16];
#pragma unroll
          for (int q = 0; q < 4; ++q) tmem_ld16(tmO + lane_base + (c0 + q) * 16, rr[q]);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
#pragma unroll
            for (int e = 0; e < 16; ++e) rr[q][e] = __float_as_uint(__uint_as_float(rr[q][e]) * alpha);
            tmem_st16(tmO + lane_base + (c0 + q) * 16, rr[q]);
          }
        }
        tmem_wait_st();
      }
      // P tile row r: 64 f16 values = 8 chunks of 16 B
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = make_uint4(pack_f16x2(pv[8 * c + 0], pv[8 * c + 1]), pack_f16x2(pv[8 * c + 2], pv[8 * c + 3]),
                                   pack_f16x2(pv[8 * c + 4], pv[8 * c + 5]), pack_f16x2(pv[8 * c + 6], pv[8 * c + 7]));
        *reinterpret_cast<uint4*>(sP + sw128_offset(r, c)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
      if (et == 0) trace(p, kTrP);
    }

    // ---- epilogue ----
    if (!waited) pdl_wait();
    if (ok && nbl > 0) ok = mbar_wait(o_full, (nbl - 1) & 1, p.status, kDevTimeoutMmaDone);
    tc_fence_after();
    if (ok && nbl > 0) {
      const bool final_out = p.splits == 1;
      const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
      const long tok = static_cast<long>(b) * p.S + s_row;
      __nv_bfloat16* orow = p.out + tok * (static_cast<long>(p.Hq) * kD) + h_row * kD;
      const long wcta = (static_cast<long>(b) * p.q_tiles + qt) * p.splits + sp;
      const long wrow = wcta * kQR + r;
      // partial O layout [cta][16-column chunk][row][16]: a warp's rows write
      // consecutive 64-byte runs (coalesced)
      float* wrow_o = p.ws_o ? p.ws_o + (wcta * (kD / 16) * kQR + r) * 16 : nullptr;
      if (et == 0) trace(p, kTrO);
#pragma unroll 1
      for (int c0 = 0; c0 < kD / 16; c0 += 4) {
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
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              *reinterpret_cast<float4*>(wrow_o + static_cast<long>(c) * kQR * 16 + 4 * e) =
                  make_float4(__uint_as_float(rr[q][4 * e]), __uint_as_float(rr[q][4 * e + 1]),
                              __uint_as_float(rr[q][4 * e + 2]), __uint_as_float(rr[q][4 * e + 3]));
          }
        }
      }
      if (!final_out && row_valid) p.ws_ml[wrow] = make_float2(m_run, l_run);
      if (et == 0) trace(p, kTrOStored);
    }
    (void)et;
  }

  tc_fence_before();
  __syncthreads();
  // drain a producer that stopped early
  if (warp == 0 && lane == 0 && issued_ctx > 0) mbar_wait(kv_full, (issued_ctx - 1) & 1, p.status, kDevTimeoutTmaFull);
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0) trace(p, kTrEnd);
}

// ------------------------------------------------------------ dense mode ---
// Pre-pass: key block j (64 keys) of stream b -> dense bf16 K / f16 V rows and
// per-key scales.  Context keys: the exact int8 -> bf16 / f16 casts with the
// per-token scales moved to the scores (K) and the probabilities (V), or the
// reference uint8 dequantize ((q - zp) * scale, rounded per op to the scale
// dtype) with unit scales; the new keys: bf16 K as is, V as f16 of its bf16
// value; keys past n_ctx / S (or masked by ctx_valid) get scale 0 and -inf.
// One CTA per 16 keys of a block (grid = 4 x blocks x streams), blocks from
// j0 on (j0 = n_ctx_blocks: only the new keys, the context rows are kept).
__global__ void __launch_bounds__(256) kv_dense_kernel(const __grid_constant__ AttnParams p, const uint8_t* k_ring,
                                                       const uint8_t* v_ring, int j0) {
  constexpr int kKeys = 16;
  pdl_wait();
  const int j = j0 + (blockIdx.x >> 2), q0 = (blockIdx.x & 3) * kKeys, b = blockIdx.y;
  const long row0 = static_cast<long>(b) * p.Lk + static_cast<long>(j) * kKB;
  const bool sbf16 = p.scale_bf16 != 0;
  __shared__ float dq[4][kKB];  // reference scheme: k scale, v scale, k zp, v zp
  if (j < p.n_ctx_blocks) {
    if (threadIdx.x < kKeys) {
      const int t = q0 + threadIdx.x;
      const long slot = static_cast<long>(j) * kKB + t;
      const long gi = static_cast<long>(b) * p.cap + (slot < p.cap ? slot : p.cap - 1);
      bool valid = slot < p.n_ctx;
      if (valid && p.ctx_valid) valid = p.ctx_valid[gi] != 0;
      p.key_add[row0 + t] = valid ? 0.f : -INFINITY;
      p.key_nb[row0 + t] = -1;
      if (p.mode == kQuantI8Sym) {
        p.key_ks[row0 + t] = valid ? static_cast<const float*>(p.k_scale)[gi] * p.scale_log2 : 0.f;
        p.key_vs[row0 + t] = valid ? static_cast<const float*>(p.v_scale)[gi] : 0.f;
      } else {
        p.key_ks[row0 + t] = valid ? p.scale_log2 : 0.f;
        p.key_vs[row0 + t] = 1.f;
        dq[0][t] = load_scalar(p.k_scale, gi, sbf16);
        dq[1][t] = load_scalar(p.v_scale, gi, sbf16);
        dq[2][t] = load_scalar(p.k_zp, gi, sbf16);
        dq[3][t] = load_scalar(p.v_zp, gi, sbf16);
      }
    }
    __syncthreads();
    // 16 keys x (K, V) x 16 chunks of 16 quantized values
    for (int it = threadIdx.x; it < 2 * kKeys * 16; it += blockDim.x) {
      const bool isv = it >= kKeys * 16;
      const int w = isv ? it - kKeys * 16 : it;
      const int key = q0 + (w >> 4), g = w & 15;
      long slot = static_cast<long>(j) * kKB + key;
      if (slot >= p.cap) slot = p.cap - 1;
      const uint4 raw = *reinterpret_cast<const uint4*>((isv ? v_ring : k_ring) +
                                                        (static_cast<long>(b) * p.cap + slot) * kD + g * 16);
      const uint8_t* b8 = reinterpret_cast<const uint8_t*>(&raw);
      float f[16];
      if (p.mode == kQuantI8Sym) {
#pragma unroll
        for (int e = 0; e < 16; ++e) f[e] = static_cast<float>(static_cast<int8_t>(b8[e]));
      } else {
        const float sc = dq[isv ? 1 : 0][key], zp = dq[isv ? 3 : 2][key];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float t = round_to(__fsub_rn(static_cast<float>(b8[e]), zp), sbf16);
          f[e] = round_to(__fmul_rn(t, sc), sbf16);
        }
      }
      uint32_t w8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) w8[e] = isv ? pack_f16x2(f[2 * e], f[2 * e + 1]) : pack_bf16x2(f[2 * e], f[2 * e + 1]);
      uint4* dst = isv ? reinterpret_cast<uint4*>(p.vd + (row0 + key) * kD + g * 16)
                       : reinterpret_cast<uint4*>(p.kd + (row0 + key) * kD + g * 16);
      dst[0] = make_uint4(w8[0], w8[1], w8[2], w8[3]);
      dst[1] = make_uint4(w8[4], w8[5], w8[6], w8[7]);
    }
  } else {
    const int nb0 = (j - p.n_ctx_blocks) * kKB;
    if (threadIdx.x < kKeys) {
      const int t = q0 + threadIdx.x;
      const int kk = nb0 + t;
      p.key_ks[row0 + t] = kk < p.S ? p.scale_log2 : 0.f;
      p.key_add[row0 + t] = kk < p.S ? 0.f : -INFINITY;
      p.key_vs[row0 + t] = 1.f;
      p.key_nb[row0 + t] = (kk < p.S && p.new_block) ? p.new_block[kk] : 0;
    }
    // 16 keys x (K, V) x 32 chunks of 8 bf16 values
    for (int it = threadIdx.x; it < 2 * kKeys * 32; it += blockDim.x) {
      const bool isv = it >= kKeys * 32;
      const int w = isv ? it - kKeys * 32 : it;
      const int key = q0 + (w >> 5), c = w & 31;
      const int kk = nb0 + key;
      uint4 raw = make_uint4(0u, 0u, 0u, 0u);
      if (kk < p.S) raw = *reinterpret_cast<const uint4*>((isv ? p.v_new : p.k_new) +
                                                           (static_cast<long>(b) * p.S + kk) * kD + c * 8);
      if (isv) {
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
        uint32_t w4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h2[e]);
          w4[e] = pack_f16x2(f.x, f.y);
        }
        *reinterpret_cast<uint4*>(p.vd + (row0 + key) * kD + c * 8) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      } else {
        *reinterpret_cast<uint4*>(p.kd + (row0 + key) * kD + c * 8) = raw;
      }
    }
  }
  pdl_launch_dependents();
}

// Attention over the dense keys in 128-key blocks.  One QK^T instruction then
// covers 128 keys (N = 128), so a 128-key block costs 16 score and 8 P.V
// instructions instead of 2 x (16 + 4) at 64 keys, and P stays in TMEM (the
// A operand of P.V), which leaves shared memory for whole 128-key K tiles.
//   Producer: Q once; per block the K tile by dim block (each of the four
//   64-dim blocks reloads as soon as the previous block's scores over it are
//   done), the block's per-key words (three stages), and V in two 64-key
//   halves (each reloads once the previous block's P.V over it is done).
//   MMA issuer: S_jl = Q K_jl^T into TMEM buffer jl % 2, then P_{jl-1} V_{jl-1}
//   into O, so the next block's scores are computed during the softmax.
//   Workers: the softmax of S_jl into P_jl (f16, written over S_jl's own
//   columns), O rescaled when the running maximum moves.
constexpr int kDKB = 128;               // keys per block
constexpr int kDOffQ = 0;               // 4 x [128 rows x 64 dims] bf16
constexpr int kDOffK = 65536;           // 4 x [128 keys x 64 dims] bf16, K-major
constexpr int kDOffV = 131072;          // 2 halves x 4 x [64 keys x 64 dims] f16, MN-major
constexpr int kDScaleWords = 4 * kDKB;  // ks, vs, kadd, nb of one block
constexpr int kDOffScale = 196608;      // 3 stages x kDScaleWords words
constexpr int kDOffBar = kDOffScale + 3 * kDScaleWords * 4;
constexpr int kDOffXchg = kDOffBar + 256;  // 768 floats: row maxima and sums of the two column halves
constexpr int kDSmemBytes = kDOffXchg + 3072 + 1024;
static_assert(kDSmemBytes <= 227 * 1024, "dense attention shared memory");
// warps 0-1 as in attention_kernel; warps 2-9 run the softmax and the
// epilogue, two per TMEM lane quadrant, each on half of a row's columns
constexpr int kDWorkers = 256;
constexpr int kDThreads = 64 + kDWorkers;

// Barrier over the two worker warps of a TMEM lane quadrant that also ANDs a
// flag over them: both warps leave a loop together when either saw a failed
// (bounded) wait, so neither waits at a named barrier for a warp that left.
__device__ __forceinline__ bool pair_all(int quad, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, 64, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u), "r"(2 + quad)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(kDThreads, 1)
    attention_dense_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
  // p.n_blocks counts 128-key blocks here
  const int blk_begin = sp * p.n_blocks / p.splits;
  const int nbl = (sp + 1) * p.n_blocks / p.splits - blk_begin;
  uint8_t* sQ = smem + kDOffQ;
  float* sScale = reinterpret_cast<float*>(smem + kDOffScale);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [4] per dim block
  uint64_t* k_empty = bars + 5;   // [4]
  uint64_t* v_full = bars + 9;    // [2] per 64-key half
  uint64_t* v_empty = bars + 11;  // [2]
  uint64_t* s_full = bars + 13;   // [2] per S buffer
  uint64_t* sc_full = bars + 15;  // [3] per scale stage
  uint64_t* p_ready = bars + 18;  // [2] per S buffer: P_jl written (blocks jl, jl + 2, ... on one barrier)
  uint64_t* o_done = bars + 20;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 21);
  if (threadIdx.x == 0) trace(p, kTrStart);
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
    }
    for (int i = 0; i < 3; ++i) mbar_init(&sc_full[i], 1);
    for (int i = 0; i < 2; ++i) mbar_init(&p_ready[i], kDWorkers / 32);
    mbar_init(o_done, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmO = tmem;  // S buffers at columns 256 and 384, P over each S's own columns
  auto tmS = [&](int jl) { return tmem + 256 + static_cast<uint32_t>(jl & 1) * kDKB; };
  pdl_launch_dependents();
  const long q_row0 = static_cast<long>(b) * p.Hq * p.S + static_cast<long>(qt) * kQR;
  int k_iss = 0, v_iss = 0;  // dim-block / half loads issued (4 / 2 per block)

  if (warp == 0) {
    pdl_wait();
    if (lane == 0 && nbl > 0) {
      mbar_arrive_expect_tx(q_full, 4 * 16384);
      for (int a = 0; a < 4; ++a) tma_load_2d(sQ + a * 16384, &tmQ, q_full, a * 64, static_cast<int>(q_row0));
      // two queues from one thread, bounded in time: K dim block a of block
      // kb once the scores of block kb-1 over it are done (with dim block 0,
      // the block's per-key words into stage kb % 3), V half h of block vb
      // once P.V of block vb-1 over it is done; V never ahead of K
      const unsigned long long t0 = globaltimer_ns();
      while (v_iss < 2 * nbl) {
        bool moved = false;
        if (k_iss < 4 * nbl) {
          const int kb = k_iss >> 2, a = k_iss & 3;
          if (kb == 0 || mbar_try_wait(&k_empty[a], (kb - 1) & 1)) {
            const long key0 = static_cast<long>(b) * p.Lk + static_cast<long>(blk_begin + kb) * kDKB;
            if (a == 0) {
              float* sc = sScale + (kb % 3) * kDScaleWords;
              mbar_arrive_expect_tx(&sc_full[kb % 3], kDScaleWords * 4);
              bulk_load(sc, p.key_ks + key0, kDKB * 4, &sc_full[kb % 3]);
              bulk_load(sc + kDKB, p.key_vs + key0, kDKB * 4, &sc_full[kb % 3]);
              bulk_load(sc + 2 * kDKB, p.key_add + key0, kDKB * 4, &sc_full[kb % 3]);
              bulk_load(sc + 3 * kDKB, p.key_nb + key0, kDKB * 4, &sc_full[kb % 3]);
            }
            mbar_arrive_expect_tx(&k_full[a], kDKB * 128);
            tma_load_2d(smem + kDOffK + a * 16384, &tmK, &k_full[a], a * 64, static_cast<int>(key0));
            ++k_iss;
            moved = true;
          }
        }
        if (v_iss < 2 * (k_iss >> 2)) {
          const int vb = v_iss >> 1, h = v_iss & 1;
          if (vb == 0 || mbar_try_wait(&v_empty[h], (vb - 1) & 1)) {
            const long key0 = static_cast<long>(b) * p.Lk + static_cast<long>(blk_begin + vb) * kDKB + h * 64;
            mbar_arrive_expect_tx(&v_full[h], 32768);
            for (int a = 0; a < 4; ++a)
              tma_load_2d(smem + kDOffV + h * 32768 + a * 8192, &tmV, &v_full[h], a * 64, static_cast<int>(key0));
            ++v_iss;
            moved = true;
          }
        }
        if (!moved && globaltimer_ns() - t0 > kWaitLimitNs) {
          record_error(p.status, kDevTimeoutStageEmpty);
          break;
        }
      }
      trace(p, kTrIssued);
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0 && nbl > 0) {
      constexpr uint32_t idesc_s = make_idesc_f16(kQR, kDKB, true);
      constexpr uint32_t idesc_o = make_idesc_f16(kQR, kD, false, true);
      bool ok = mbar_wait(q_full, 0, p.status, kDevTimeoutTmaFull);
      auto pv = [&](int jp) {  // O += P_jp V_jp, P from TMEM
        if (!(ok = mbar_wait(&p_ready[jp & 1], (jp >> 1) & 1, p.status, kDevTimeoutConvert))) return;
        tc_fence_after();
        for (int h = 0; h < 2 && ok; ++h) {
          if (!(ok = mbar_wait(&v_full[h], jp & 1, p.status, kDevTimeoutTmaFull))) return;
          tc_fence_after();
          const uint32_t v_base = smem_u32(smem + kDOffV + h * 32768);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t bd = make_sdesc_sw128(v_base + ks * 2048, 8192, 1024);
            umma_f16_ts(tmO, tmS(jp) + static_cast<uint32_t>(h * 64 + ks * 8), bd, idesc_o,
                        (jp > 0 || h > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(&v_empty[h]);
        }
        umma_commit(o_done);
      };
      for (int jl = 0; jl < nbl && ok; ++jl) {
        // S buffer jl % 2 last held P_{jl-2}, read by the P.V issued before
        // this point (tcgen05.mma of one thread run in order)
        for (int a = 0; a < 4 && ok; ++a) {
          if (!(ok = mbar_wait(&k_full[a], jl & 1, p.status, kDevTimeoutTmaFull))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = make_sdesc_sw128(smem_u32(sQ + a * 16384) + kk * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(smem_u32(smem + kDOffK + a * 16384) + kk * 32, 16, 1024);
            umma_f16_ss(tmS(jl), ad, bd, idesc_s, (a > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&k_empty[a]);  // this dim block may be reloaded
        }
        if (!ok) break;
        umma_commit(&s_full[jl & 1]);
        if (jl >= 1) pv(jl - 1);
      }
      if (ok) pv(nbl - 1);
    }
  } else {
    pdl_wait();
    const int quad = warp & 3;
    const int ch = (threadIdx.x - 64) >> 7;  // this warp's half of the row: 64 score / 128 output columns
    const int r = quad * 32 + lane;          // query row inside the tile == TMEM lane
    float* mx_x = reinterpret_cast<float*>(smem + kDOffXchg);  // [2 blocks][2 halves][128] row maxima
    float* l_x = mx_x + 512;                                   // [2 halves][128] row sums
    const int R = qt * kQR + r;
    const bool row_valid = R < p.Hq * p.S;
    const int s_row = row_valid ? R % p.S : 0;
    const int h_row = row_valid ? R / p.S : 0;
    const int my_block = (row_valid && p.new_block) ? p.new_block[s_row] : 0;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    constexpr int kHalf = kDKB / 2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int jl = 0; jl < nbl; ++jl) {
      if (ok) ok = mbar_wait(&sc_full[jl % 3], (jl / 3) & 1, p.status, kDevTimeoutTmaFull);
      if (ok) ok = mbar_wait(&s_full[jl & 1], (jl >> 1) & 1, p.status, kDevTimeoutMmaDone);
      ok = __all_sync(0xffffffffu, ok);
      // this half's keys: score scale (log2 units), value scale, additive
      // mask and block id (context keys -1: always visible)
      const float* sc = sScale + (jl % 3) * kDScaleWords + kHalf * ch;
      const float* ks_s = sc;
      const float* vs_s = sc + kDKB;
      const float* kadd_s = sc + 2 * kDKB;
      const int* nb_s = reinterpret_cast<const int*>(sc + 3 * kDKB);
      float z[kHalf];
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (ok) {
        tc_fence_after();
        {
          uint32_t rr[4][16];
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld16(tmS(jl) + lane_base + kHalf * ch + 16 * c, rr[c]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 16; ++e) z[c * 16 + e] = __uint_as_float(rr[c][e]);
        }
#pragma unroll
        for (int c = 0; c < kHalf / 4; ++c) {
          const float4 km = reinterpret_cast<const float4*>(ks_s)[c];
          const float4 ka = reinterpret_cast<const float4*>(kadd_s)[c];
          z[4 * c + 0] = fmaf(z[4 * c + 0], km.x, ka.x);
          z[4 * c + 1] = fmaf(z[4 * c + 1], km.y, ka.y);
          z[4 * c + 2] = fmaf(z[4 * c + 2], km.z, ka.z);
          z[4 * c + 3] = fmaf(z[4 * c + 3], km.w, ka.w);
          if (p.new_block) {  // new key j is visible to row i iff new_block[j] <= new_block[i]
            const int4 nb = reinterpret_cast<const int4*>(nb_s)[c];
            if (nb.x > my_block) z[4 * c + 0] = -INFINITY;
            if (nb.y > my_block) z[4 * c + 1] = -INFINITY;
            if (nb.z > my_block) z[4 * c + 2] = -INFINITY;
            if (nb.w > my_block) z[4 * c + 3] = -INFINITY;
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) mx[e] = fmaxf(mx[e], z[4 * c + e]);
        }
      }
      // the row's max over both column halves (the partner warp holds the other)
      float* mxb = mx_x + (jl & 1) * 256;
      mxb[ch * 128 + r] = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      ok = pair_all(quad, ok);
      if (!ok) break;  // both warps of the pair agree
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
      if (__any_sync(0xffffffffu, need)) {
        // O is final for the rescale once P_{jl-1} V_{jl-1} is done (need
        // implies jl >= 1; a failed wait skips the rest of this block and the
        // pair leaves the loop together at the next exchange)
        ok = __all_sync(0xffffffffu, mbar_wait(o_done, (jl - 1) & 1, p.status, kDevTimeoutMmaDone));
        if (!ok) continue;
        tc_fence_after();
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
      }
      // P (times the value scales) as f16 pairs over the first 32 of this
      // half's 64 score columns, which are already read
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int hq = 0; hq < 2; ++hq) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 8 * hq; c < 8 * hq + 8; ++c) {
          const float4 vsc = reinterpret_cast<const float4*>(vs_s)[c];
          const float vv[4] = {vsc.x, vsc.y, vsc.z, vsc.w};
          float pe[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            pe[e] = ex2_approx(z[4 * c + e] - m_sub);
            ps[e] += pe[e];
            pe[e] *= vv[e];
          }
          pk[(2 * c) & 15] = pack_f16x2(pe[0], pe[1]);
          pk[(2 * c + 1) & 15] = pack_f16x2(pe[2], pe[3]);
        }
        tmem_st16(tmS(jl) + lane_base + kHalf * ch + 16 * hq, pk);
      }
      l_run = l_run * alpha + ((ps[0] + ps[1]) + (ps[2] + ps[3]));
      m_run = m_use;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[jl & 1]);
    }
    // ---- epilogue (the layout of attention_kernel's) ----
    if (ok && nbl > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_done, (nbl - 1) & 1, p.status, kDevTimeoutMmaDone));
    tc_fence_after();
    // the row sum over both halves, in a fixed order (every pair takes this
    // barrier once, whatever happened in the loop)
    if (nbl > 0) {
      l_x[ch * 128 + r] = l_run;
      ok = pair_all(quad, ok);
    }
    if (ok && nbl > 0) {
      const bool final_out = p.splits == 1;
      l_run = l_x[r] + l_x[128 + r];
      const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
      const long tok = static_cast<long>(b) * p.S + s_row;
      __nv_bfloat16* orow = p.out + tok * (static_cast<long>(p.Hq) * kD) + h_row * kD;
      const long wcta = (static_cast<long>(b) * p.q_tiles + qt) * p.splits + sp;
      float* wrow_o = p.ws_o ? p.ws_o + (wcta * (kD / 16) * kQR + r) * 16 : nullptr;
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
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              *reinterpret_cast<float4*>(wrow_o + static_cast<long>(c) * kQR * 16 + 4 * e) =
                  make_float4(__uint_as_float(rr[q][4 * e]), __uint_as_float(rr[q][4 * e + 1]),
                              __uint_as_float(rr[q][4 * e + 2]), __uint_as_float(rr[q][4 * e + 3]));
          }
        }
      }
      if (!final_out && row_valid && ch == 0) p.ws_ml[wcta * kQR + r] = make_float2(m_run, l_run);
    }
  }
  tc_fence_before();
  __syncthreads();
  // every issued load completes before the block leaves (a producer or MMA
  // issuer that stopped early)
  if (warp == 0 && lane == 0) {
    for (int a = 0; a < 4; ++a) {
      const int n = (k_iss - a + 3) / 4;
      if (n > 0) mbar_wait(&k_full[a], (n - 1) & 1, p.status, kDevTimeoutTmaFull);
    }
    for (int h = 0; h < 2; ++h) {
      const int n = (v_iss - h + 1) / 2;
      if (n > 0) mbar_wait(&v_full[h], (n - 1) & 1, p.status, kDevTimeoutTmaFull);
    }
    const int n_sc = (k_iss + 3) / 4;
    for (int s = 0; s < 3; ++s) {
      const int n = (n_sc - s + 2) / 3;
      if (n > 0) mbar_wait(&sc_full[s], (n - 1) & 1, p.status, kDevTimeoutTmaFull);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0) trace(p, kTrEnd);
}

// Merges the kv_splits partial results of every query row: one warp per row,
// lane l holding 8 of the 256 columns.  Split s's (m, l) sits in lane s (at
// most 32 splits), so the row max and the weights 2^(m_s - M) are a warp
// reduction and broadcasts; the first 8 splits' partials are requested before
// the (m, l) arrive, so the two loads overlap.
__global__ void __launch_bounds__(128) attention_combine_kernel(const AttnParams p) {
  pdl_wait();
  const long g = static_cast<long>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long rows = static_cast<long>(p.B) * p.q_tiles * kQR;
  if (g < rows) {
    const int r = static_cast<int>(g % kQR);
    const int qt = static_cast<int>((g / kQR) % p.q_tiles);
    const int b = static_cast<int>(g / (static_cast<long>(kQR) * p.q_tiles));
    const int R = qt * kQR + r;
    if (R < p.Hq * p.S) {
      const long base = (static_cast<long>(b) * p.q_tiles + qt) * p.splits;
      constexpr int kBatch = 8;
      auto load = [&](int s, float4& a, float4& c) {
        const float* o = p.ws_o + (((base + s) * (kD / 16) + (lane >> 1)) * kQR + r) * 16 + (lane & 1) * 8;
        a = *reinterpret_cast<const float4*>(o);
        c = *reinterpret_cast<const float4*>(o + 4);
      };
      float4 a[kBatch], c[kBatch];
#pragma unroll
      for (int q = 0; q < kBatch; ++q)
        if (q < p.splits) load(q, a[q], c[q]);
      const float2 ml = lane < p.splits ? p.ws_ml[(base + lane) * kQR + r] : make_float2(-INFINITY, 0.f);
      const bool live = ml.x != -INFINITY && ml.y > 0.f;
      const float M = warp_max(live ? ml.x : -INFINITY);
      const float w = live ? exp2f(ml.x - M) : 0.f;
      const float L = warp_sum(w * ml.y);
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int s0 = 0; s0 < p.splits; s0 += kBatch) {
        if (s0 > 0) {
#pragma unroll
          for (int q = 0; q < kBatch; ++q)
            if (s0 + q < p.splits) load(s0 + q, a[q], c[q]);
        }
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
          const float ws = __shfl_sync(0xffffffffu, w, (s0 + q) & 31);
          if (s0 + q >= p.splits) continue;
          acc[0] = fmaf(ws, a[q].x, acc[0]); acc[1] = fmaf(ws, a[q].y, acc[1]);
          acc[2] = fmaf(ws, a[q].z, acc[2]); acc[3] = fmaf(ws, a[q].w, acc[3]);
          acc[4] = fmaf(ws, c[q].x, acc[4]); acc[5] = fmaf(ws, c[q].y, acc[5]);
          acc[6] = fmaf(ws, c[q].z, acc[6]); acc[7] = fmaf(ws, c[q].w, acc[7]);
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      const int s_row = R % p.S, h_row = R / p.S;
      __nv_bfloat16* orow =
          p.out + (static_cast<long>(b) * p.S + s_row) * (static_cast<long>(p.Hq) * kD) + h_row * kD + lane * 8;
      *reinterpret_cast<uint4*>(orow) = make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv),
                                                   pack_bf16x2(acc[2] * inv, acc[3] * inv),
                                                   pack_bf16x2(acc[4] * inv, acc[5] * inv),
                                                   pack_bf16x2(acc[6] * inv, acc[7] * inv));
    }
  }
  pdl_launch_dependents();
}

struct Geometry {
  int q_tiles, n_ctx_blocks, n_blocks, splits;
};

int geometry(const rfx_attn_desc& d, Geometry* g) {
  if (d.B < 1 || d.num_q_heads < 1 || d.head_dim != kD || d.S < 1 || d.capacity < 0 || d.n_ctx < 0 ||
      d.n_ctx > d.capacity)
    return set_error(RFX_E_INVAL, "rfx_attention: need head_dim=256, S>=1, 0<=n_ctx<=capacity");
  if (d.quant_mode != RFX_QUANT_I8_SYM && d.quant_mode != RFX_QUANT_U8_REF)
    return set_error(RFX_E_INVAL, "rfx_attention: quant_mode");
  if (d.kv_source != RFX_KV_RING_TILES && d.kv_source != RFX_KV_DENSE)
    return set_error(RFX_E_INVAL, "rfx_attention: kv_source");
  g->q_tiles = (d.num_q_heads * d.S + kQR - 1) / kQR;
  g->n_ctx_blocks = (d.n_ctx + kKB - 1) / kKB;
  g->n_blocks = g->n_ctx_blocks + (d.S + kKB - 1) / kKB;
  // the dense attention walks 128-key blocks: the conversion pads the keys to
  // an even number of 64-key blocks (the padding keys are masked)
  const bool dense = d.kv_source == RFX_KV_DENSE;
  if (dense) g->n_blocks += g->n_blocks & 1;
  const int att_blocks = dense ? g->n_blocks / 2 : g->n_blocks;
  int nsm = 148;
  rfx_num_sms(&nsm);
  int splits = d.kv_splits;
  if (splits <= 0) {
    const int ctas = d.B * g->q_tiles;
    splits = std::max(1, std::min(att_blocks, nsm / std::max(1, ctas)));
  }
  if (splits > att_blocks) splits = att_blocks;
  if (splits > 32) splits = 32;  // the combine kernel merges at most 32 partials per row
  g->splits = splits;
  return RFX_OK;
}

}  // namespace

namespace {
// Workspace: the split-KV partials (O, then (m, l)), then in dense mode the
// dense keys at 1024-byte aligned offsets: bf16 K, f16 V [B][Lk][D] and the
// per-key ks, vs, kadd [B][Lk] fp32 and block ids [B][Lk] int32.
struct WsLayout {
  size_t partials, kd, vd, ks, vs, kadd, nb, total;
};
WsLayout ws_layout(const rfx_attn_desc& d, const Geometry& g) {
  WsLayout w{};
  const size_t rows = static_cast<size_t>(d.B) * g.q_tiles * g.splits * kQR;
  w.partials = g.splits > 1 ? rows * kD * sizeof(float) + rows * sizeof(float2) : 0;
  size_t off = (w.partials + 1023) & ~size_t(1023);
  if (d.kv_source == RFX_KV_DENSE) {
    const size_t keys = static_cast<size_t>(d.B) * g.n_blocks * kKB;
    auto take = [&](size_t bytes) {
      const size_t o = off;
      off = (off + bytes + 1023) & ~size_t(1023);
      return o;
    };
    w.kd = take(keys * kD * 2);
    w.vd = take(keys * kD * 2);
    w.ks = take(keys * 4);
    w.vs = take(keys * 4);
    w.kadd = take(keys * 4);
    w.nb = take(keys * 4);
    w.total = off;
  } else {
    w.total = w.partials;
  }
  return w;
}
}  // namespace

size_t attention_workspace_bytes(const rfx_attn_desc& d) {
  Geometry g;
  if (geometry(d, &g) != RFX_OK) return 0;
  return ws_layout(d, g).total;
}

int attention_launches(const rfx_attn_desc& d) {
  Geometry g;
  if (geometry(d, &g) != RFX_OK) return 0;
  return (d.kv_source == RFX_KV_DENSE ? 1 : 0) + 1 + (g.splits > 1 ? 1 : 0);
}

int build_attention_maps(const rfx_attn_desc& d, CUtensorMap* tmQ, CUtensorMap* tmK, CUtensorMap* tmV) {
  Geometry g;
  int rc = geometry(d, &g);
  if (rc) return rc;
  if (!d.q || !d.k_new || !d.v_new || !d.out) return set_error(RFX_E_INVAL, "rfx_attention: null q/k_new/v_new/out");
  const uint64_t qrows = static_cast<uint64_t>(d.B) * d.num_q_heads * d.S;
  rc = make_tmap_2d(tmQ, d.q, 2, kD, qrows, kD * 2, 64, kQR, true);
  if (rc) return rc;
  if (d.n_ctx > 0 && (!d.k_ring || !d.v_ring || !d.k_scale || !d.v_scale ||
                     (d.quant_mode == RFX_QUANT_U8_REF && (!d.k_zp || !d.v_zp))))
    return set_error(RFX_E_INVAL, "rfx_attention: null ring/scale pointers");
  if (d.kv_source == RFX_KV_DENSE) {
    // the dense keys live in the workspace: its size and alignment are checked here
    const WsLayout w = ws_layout(d, g);
    if (!d.workspace || d.workspace_bytes < w.total || (reinterpret_cast<uintptr_t>(d.workspace) & 1023u))
      return set_error(RFX_E_INVAL, "rfx_attention: RFX_KV_DENSE needs a 1024-byte aligned workspace of %zu bytes",
                       w.total);
    const uint64_t keys = static_cast<uint64_t>(d.B) * g.n_blocks * kKB;
    char* ws = static_cast<char*>(d.workspace);
    rc = make_tmap_2d(tmK, ws + w.kd, 2, kD, keys, kD * 2, 64, kDKB, true);  // 128-key K tiles
    if (rc) return rc;
    return make_tmap_2d(tmV, ws + w.vd, 2, kD, keys, kD * 2, 64, kKB, true);   // 64-key V halves
  }
  if (d.n_ctx > 0) {
    const uint64_t krows = static_cast<uint64_t>(d.B) * d.capacity;
    rc = make_tmap_2d(tmK, d.k_ring, 1, kD, krows, kD, kD, kKB, false);
    if (rc) return rc;
    rc = make_tmap_2d(tmV, d.v_ring, 1, kD, krows, kD, kD, kKB, false);
    if (rc) return rc;
  } else {
    *tmK = *tmQ;
    *tmV = *tmQ;
  }
  return RFX_OK;
}

int launch_attention(const rfx_attn_desc& d, const CUtensorMap* tmQ, const CUtensorMap* tmK, const CUtensorMap* tmV,
                     cudaStream_t stream, bool pdl) {
  Geometry g;
  int rc = geometry(d, &g);
  if (rc) return rc;
  const WsLayout wl = ws_layout(d, g);
  const size_t need = wl.total;
  const bool dense = d.kv_source == RFX_KV_DENSE;
  if (need > 0 && (!d.workspace || d.workspace_bytes < need ||
                   (reinterpret_cast<uintptr_t>(d.workspace) & (dense ? 1023u : 15u))))
    return set_error(RFX_E_INVAL, "rfx_attention: workspace of %zu bytes (%d-byte aligned) required", need,
                     dense ? 1024 : 16);
  const void* fn =
      dense ? reinterpret_cast<const void*>(attention_dense_kernel) : reinterpret_cast<const void*>(attention_kernel);
  const int smem_bytes = dense ? kDSmemBytes : kSmemBytes;
  rc = ensure_smem_attr(fn, smem_bytes);
  if (rc) return rc;

  AttnParams p{};
  p.B = d.B;
  p.Hq = d.num_q_heads;
  p.S = d.S;
  p.cap = d.capacity;
  p.n_ctx = d.n_ctx;
  p.mode = d.quant_mode;
  p.scale_bf16 = d.scale_dtype == RFX_DTYPE_BF16;
  p.q_tiles = g.q_tiles;
  p.splits = g.splits;
  p.n_ctx_blocks = g.n_ctx_blocks;
  p.n_blocks = dense ? g.n_blocks / 2 : g.n_blocks;  // attention blocks: 128 keys (dense) or 64
  p.k_new = static_cast<const __nv_bfloat16*>(d.k_new);
  p.v_new = static_cast<const __nv_bfloat16*>(d.v_new);
  p.k_scale = d.k_scale;
  p.v_scale = d.v_scale;
  p.k_zp = d.k_zp;
  p.v_zp = d.v_zp;
  p.ctx_valid = d.ctx_valid;
  p.new_block = d.new_block;
  p.scale_log2 = d.softmax_scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(d.out);
  if (wl.partials > 0) {
    p.ws_o = static_cast<float*>(d.workspace);
    const size_t rows = static_cast<size_t>(d.B) * g.q_tiles * g.splits * kQR;
    p.ws_ml = reinterpret_cast<float2*>(static_cast<char*>(d.workspace) + rows * kD * sizeof(float));
  }
  if (dense) {
    char* ws = static_cast<char*>(d.workspace);
    p.kd = reinterpret_cast<__nv_bfloat16*>(ws + wl.kd);
    p.vd = reinterpret_cast<__half*>(ws + wl.vd);
    p.key_ks = reinterpret_cast<float*>(ws + wl.ks);
    p.key_vs = reinterpret_cast<float*>(ws + wl.vs);
    p.key_add = reinterpret_cast<float*>(ws + wl.kadd);
    p.key_nb = reinterpret_cast<int*>(ws + wl.nb);
    p.Lk = g.n_blocks * kKB;
  }
  p.status = device_status_ptr();
  p.trace = static_cast<unsigned long long*>(trace_buffer(static_cast<size_t>(g.q_tiles) * g.splits * d.B * 16));

  CUtensorMap q = *tmQ, k = *tmK, v = *tmV;
  if (dense) {
    const uint8_t* kr = static_cast<const uint8_t*>(d.k_ring);
    const uint8_t* vr = static_cast<const uint8_t*>(d.v_ring);
    int j0 = d.dense_ctx_ready ? g.n_ctx_blocks : 0;
    rc = launch_kernel(reinterpret_cast<const void*>(kv_dense_kernel), dim3(4 * (g.n_blocks - j0), d.B), dim3(256), 0,
                       stream, pdl, 1, p, kr, vr, j0);
    if (rc) return rc;
  }
  dim3 grid(g.q_tiles, g.splits, d.B);
  rc = launch_kernel(fn, grid, dim3(dense ? kDThreads : kThreads), smem_bytes, stream, pdl, 1, q, k, v, p);
  if (rc || g.splits == 1) return rc;
  const long rows = static_cast<long>(d.B) * g.q_tiles * kQR;
  dim3 cgrid(static_cast<unsigned>((rows + 3) / 4));
  return launch_kernel(reinterpret_cast<const void*>(attention_combine_kernel), cgrid, dim3(128), 0, stream, pdl, 1,
                       p);
}

// ------------------------------------------------- no-allocation variant ---
// Scratch for rfx_attention_noalloc: a file-scope device array, so the call
// never allocates.  It is for hosts that may not allocate device memory once
// they run: a controller whose memory pool reserves every device byte at
// start-up, or a real-time loop that treats any later cudaMalloc (which can
// synchronize the device and has no bounded latency) as a fault.
// The usable part starts at the first 1024-byte boundary inside the array
// (the dense key tiles need that alignment) and is kNoAllocUsableBytes long
// wherever the linker places the array.  The ring-tile source keeps only the
// split-KV partials there: B * q_tiles * kv_splits <= 63 CTAs at 132,096
// bytes each.  The dense source also keeps its bf16 K / f16 V copy of the
// keys there (1,040 bytes per key and stream).  Nothing in it has to start at
// zero: every byte a call reads was written earlier in the same call.  The
// array is shared by all calls on a device, so two calls whose launches can
// overlap (different streams, or host threads racing on one device) corrupt
// each other's data; the caller orders them.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr size_t kNoAllocUsableBytes = kNoAllocScratchBytes - 1024;
static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];
std::mutex g_scratch_mu;
std::unordered_map<int, void*> g_scratch_ptrs;

// 1024-byte aligned start of the scratch array on the current device, looked
// up once per device (cudaGetSymbolAddress with that device current).  The
// first call on a device can load the module's device code (lazy loading),
// so it belongs before any stream capture.
int noalloc_scratch(void** out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "rfx_attention_noalloc: cudaGetDevice");
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  auto it = g_scratch_ptrs.find(dev);
  if (it != g_scratch_ptrs.end()) {
    *out = it->second;
    return RFX_OK;
  }
  void* p = nullptr;
  rc = check_cuda(cudaGetSymbolAddress(&p, g_attn_scratch), "rfx_attention_noalloc: cudaGetSymbolAddress(scratch)");
  if (rc) return rc;
  const uintptr_t a = (reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023);
  void* aligned = reinterpret_cast<void*>(a);
  g_scratch_ptrs[dev] = aligned;
  *out = aligned;
  return RFX_OK;
}
}  // namespace

}  // namespace rfx

extern "C" int rfx_attention_noalloc(const rfx_attn_desc* desc, void* stream) {
  using namespace rfx;
  if (!desc) return set_error(RFX_E_INVAL, "rfx_attention_noalloc: null descriptor");
  Geometry g;
  int rc = geometry(*desc, &g);
  if (rc) return rc;
  rfx_attn_desc d = *desc;
  d.dense_ctx_ready = 0;  // the scratch is shared by every call: always convert the whole context
  size_t need = attention_workspace_bytes(d);
  if (desc->kv_splits <= 0) {
    // automatic split count: the largest one (up to the automatic choice)
    // whose scratch fits
    int splits = g.splits;
    while (need > kNoAllocUsableBytes && splits > 1) {
      d.kv_splits = --splits;
      need = attention_workspace_bytes(d);
    }
    d.kv_splits = splits;
  }
  if (need > kNoAllocUsableBytes)
    return set_error(RFX_E_INVAL,
                     "rfx_attention_noalloc: this shape needs %zu bytes of scratch, the static scratch holds %zu; "
                     "lower kv_splits or call rfx_attention with a workspace",
                     need, kNoAllocUsableBytes);
  d.workspace = nullptr;
  d.workspace_bytes = 0;
  if (need > 0) {
    rc = noalloc_scratch(&d.workspace);
    if (rc) return rc;
    d.workspace_bytes = kNoAllocUsableBytes;
  }
  CUtensorMap q, k, v;
  rc = build_attention_maps(d, &q, &k, &v);
  if (rc) return rc;
  return launch_attention(d, &q, &k, &v, static_cast<cudaStream_t>(stream), pdl_enabled());
}

extern "C" int rfx_attention_workspace_size(const rfx_attn_desc* desc, size_t* bytes) {
  using namespace rfx;
  if (!desc || !bytes) return set_error(RFX_E_INVAL, "rfx_attention_workspace_size: null argument");
  Geometry g;
  int rc = geometry(*desc, &g);
  if (rc) return rc;
  *bytes = attention_workspace_bytes(*desc);
  return RFX_OK;
}

extern "C" int rfx_attention(const rfx_attn_desc* desc, void* stream) {
  using namespace rfx;
  if (!desc) return set_error(RFX_E_INVAL, "rfx_attention: null descriptor");
  CUtensorMap q, k, v;
  int rc = build_attention_maps(*desc, &q, &k, &v);
  if (rc) return rc;
  return launch_attention(*desc, &q, &k, &v, static_cast<cudaStream_t>(stream), pdl_enabled());
}
