// Small kernels around the action expert: timestep conditioning, AdaRMSNorm
// modulation, action in-projection and the fused Euler tail.  All of them are
// HBM- or latency-bound; weights are read with 128-bit coalesced loads, one
// warp per output row, and reduced with warp shuffles.
#include "rfx_internal.h"

#include <algorithm>

namespace rfx {
namespace {

constexpr int kMaxRows = 16;  // conditioning rows (timesteps x streams) per launch

__device__ __forceinline__ float silu(float x) { return x / (1.f + expf(-x)); }

// emb[i][j]: sin for j < W/2, cos for j >= W/2, of t[i] * 2*pi / period_j with
// period_j = min_period * (max_period/min_period)^(j/(W/2-1)), all in fp64,
// rounded once to bf16 (reflex/policies/pi05/utils.py:109-121).
__global__ void sinusoid_kernel(const float* __restrict__ t, int n_t, int width, double min_period,
                                double max_period, __nv_bfloat16* __restrict__ emb) {
  pdl_wait();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int half = width / 2;
  if (idx < n_t * half) {
    const int i = idx / half, j = idx % half;
    // torch.linspace(0, 1, half) in fp64: start + step*j for the first half,
    // end - step*(half-1-j) for the second half
    const double step = half > 1 ? 1.0 / static_cast<double>(half - 1) : 0.0;
    const double frac = j < half / 2 ? step * j : 1.0 - step * (half - 1 - j);
    const double period = min_period * pow(max_period / min_period, frac);
    const double x = (1.0 / period * 2.0 * 3.141592653589793) * static_cast<double>(t[i]);
    double s, c;
    sincos(x, &s, &c);
    emb[static_cast<long>(i) * width + j] = __double2bfloat16(s);
    emb[static_cast<long>(i) * width + half + j] = __double2bfloat16(c);
  }
  pdl_launch_dependents();
}

// out[i][o] = bf16(silu(bf16(sum_k in[i][k] * W[o][k] + b[o]))) for bf16 W.
__global__ void __launch_bounds__(256) gemv_bf16_silu_kernel(const __nv_bfloat16* __restrict__ in, int n_rows,
                                                             int width, const __nv_bfloat16* __restrict__ W,
                                                             const __nv_bfloat16* __restrict__ bias, int n_out,
                                                             __nv_bfloat16* __restrict__ out) {
  extern __shared__ float xin[];  // [n_rows][width]
  pdl_wait();
  // 16-byte loads, all of a thread's loads issued before any is used
  for (int i = threadIdx.x * 8; i < n_rows * width; i += blockDim.x * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(in + i);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h2[e]);
      xin[i + 2 * e] = f.x;
      xin[i + 2 * e + 1] = f.y;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o = blockIdx.x * 8 + warp;
  if (o < n_out) {
    float acc[kMaxRows];
#pragma unroll
    for (int r = 0; r < kMaxRows; ++r) acc[r] = 0.f;
    const __nv_bfloat16* wr = W + static_cast<long>(o) * width;
    for (int k0 = 0; k0 < width; k0 += 1024) {
      uint4 wv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int k = k0 + q * 256 + lane * 8;
        if (k < width) wv[q] = *reinterpret_cast<const uint4*>(wr + k);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int k = k0 + q * 256 + lane * 8;
        if (k >= width) continue;
        const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv[q]);
        float w[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f = __bfloat1622float2(w2[e]);
          w[2 * e] = f.x;
          w[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int r = 0; r < kMaxRows; ++r) {
          if (r < n_rows) {
            const float* xr = xin + r * width + k;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[r] = fmaf(w[e], xr[e], acc[r]);
          }
        }
      }
    }
    const float bo = bias ? __bfloat162float(bias[o]) : 0.f;
#pragma unroll
    for (int r = 0; r < kMaxRows; ++r) {
      if (r < n_rows) {
        const float s = warp_sum(acc[r]);
        if (lane == 0) out[static_cast<long>(r) * n_out + o] = __float2bfloat16_rn(silu(bf16_round(s + bo)));
      }
    }
  }
  pdl_launch_dependents();
}

// AdaRMSNorm modulation: m[r][row] = sum_k cond[r][k] * W[row][k] + bias[row]
// for fp32 W [n_norms * out][width] and every conditioning row r (the Euler
// steps' timestep embeddings), in one pass over W.
//
// Every warp takes four consecutive output rows at a time (grid-stride over
// all rows) against KR conditioning rows held in shared memory as fp32, rows
// n_rows..KR-1 zero; one 16-byte shared load feeds 16 FMAs.  Lane l
// accumulates k = q*128 + 4l .. 4l+3 for q = 0, 1, ... in order.  The 16 lane
// partials of each row are then reduce-scattered across the warp (16 shuffles
// per row): lanes 2i and 2i+1 end with the sum for conditioning row
// rmap(i), and lane 2i stores it for all four rows as one float4.
__device__ __forceinline__ float halve_slots(float keep_lo, float keep_hi, bool hi, int offset) {
  const float keep = hi ? keep_hi : keep_lo;
  const float send = hi ? keep_lo : keep_hi;
  return keep + __shfl_xor_sync(0xffffffffu, send, offset);
}

// v[0..15] per lane -> sum over the warp of v[r] where
// r = 8*bit4(lane) + 4*bit3(lane) + 2*bit2(lane) + bit1(lane).
__device__ __forceinline__ float reduce_scatter16(const float (&v)[16], int lane) {
  float s8[8], s4[4], s2[2];
#pragma unroll
  for (int i = 0; i < 8; ++i) s8[i] = halve_slots(v[i], v[i + 8], lane & 16, 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) s4[i] = halve_slots(s8[i], s8[i + 4], lane & 8, 8);
#pragma unroll
  for (int i = 0; i < 2; ++i) s2[i] = halve_slots(s4[i], s4[i + 2], lane & 4, 4);
  const float s1 = halve_slots(s2[0], s2[1], lane & 2, 2);
  return s1 + __shfl_xor_sync(0xffffffffu, s1, 1);
}

template <int KR>
__global__ void __launch_bounds__(256, 2) modulation_kernel(const float* __restrict__ W, const float* __restrict__ bias,
                                                            const __nv_bfloat16* __restrict__ cond, int n_rows,
                                                            int width, int n_norms, int out_per_norm, int mode,
                                                            float* __restrict__ a2, float* __restrict__ b2,
                                                            float* __restrict__ gate) {
  static_assert(KR <= 16, "the reduce-scatter serves 16 conditioning rows");
  extern __shared__ __align__(16) float cin[];  // [KR][width]
  pdl_wait();
  for (int i = threadIdx.x * 4; i < KR * width; i += blockDim.x * 4) {
    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < n_rows * width) {
      const uint2 raw = *reinterpret_cast<const uint2*>(cond + i);
      const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
      const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
      f = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    *reinterpret_cast<float4*>(cin + i) = f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = n_norms * out_per_norm;
  constexpr int RW = 4;  // weight rows per warp iteration
  const int r_mine = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
  for (int row0 = (blockIdx.x * 8 + warp) * RW; row0 < total; row0 += gridDim.x * 8 * RW) {
    float acc[RW][KR];
#pragma unroll
    for (int j = 0; j < RW; ++j)
#pragma unroll
      for (int r = 0; r < KR; ++r) acc[j][r] = 0.f;
    const float* wr = W + static_cast<long>(row0) * width;
#pragma unroll 1
    for (int k0 = 0; k0 < width; k0 += 512) {
      // four rows' 2 KB slices are requested before any of them is used
      float4 v[RW][4];
#pragma unroll
      for (int j = 0; j < RW; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int k = k0 + q * 128 + lane * 4;
          v[j][q] = k < width ? __ldcs(reinterpret_cast<const float4*>(wr + static_cast<long>(j) * width + k))
                              : make_float4(0.f, 0.f, 0.f, 0.f);  // streamed once per chunk
        }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int k = min(k0 + q * 128 + lane * 4, width - 4);
#pragma unroll
        for (int r = 0; r < KR; ++r) {
          const float4 x = *reinterpret_cast<const float4*>(cin + r * width + k);
#pragma unroll
          for (int j = 0; j < RW; ++j) {
            acc[j][r] = fmaf(v[j][q].x, x.x, acc[j][r]);
            acc[j][r] = fmaf(v[j][q].y, x.y, acc[j][r]);
            acc[j][r] = fmaf(v[j][q].z, x.z, acc[j][r]);
            acc[j][r] = fmaf(v[j][q].w, x.w, acc[j][r]);
          }
        }
      }
    }
    float m[RW];
#pragma unroll
    for (int j = 0; j < RW; ++j) {
      float vals[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) vals[r] = r < KR ? acc[j][r] : 0.f;
      m[j] = __fadd_rn(reduce_scatter16(vals, lane), bias[row0 + j]);
    }
    if ((lane & 1) || r_mine >= n_rows) continue;
    // the four rows share one norm and one part: out_per_norm and width are multiples of 4
    const int n = row0 / out_per_norm, o = row0 - n * out_per_norm;
    const long base = (static_cast<long>(r_mine) * n_norms + n) * width;
    if (mode == RFX_ADARMS_GATE) {
      *reinterpret_cast<float4*>(a2 + base + o) = make_float4(m[0], m[1], m[2], m[3]);
      if (b2) *reinterpret_cast<float4*>(b2 + base + o) = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(gate + base + o) =
          make_float4(bf16_round(m[0]), bf16_round(m[1]), bf16_round(m[2]), bf16_round(m[3]));
    } else {
      const int part = o / width, f = o - part * width;
      if (part == 0)
        *reinterpret_cast<float4*>(a2 + base + f) =
            make_float4(__fadd_rn(1.f, m[0]), __fadd_rn(1.f, m[1]), __fadd_rn(1.f, m[2]), __fadd_rn(1.f, m[3]));
      else if (part == 1)
        *reinterpret_cast<float4*>(b2 + base + f) = make_float4(m[0], m[1], m[2], m[3]);
      else
        *reinterpret_cast<float4*>(gate + base + f) =
            make_float4(bf16_round(m[0]), bf16_round(m[1]), bf16_round(m[2]), bf16_round(m[3]));
    }
  }
  pdl_launch_dependents();
}

// h_next[row(b,s)][o] = bf16(sum_a bf16(x[b][s][a]) * W_in[o][a] + b_in[o]); one CTA per (b, s).
__device__ __forceinline__ void action_in_row(const float* xs, int A, int width, const __nv_bfloat16* __restrict__ W_in,
                                              const __nv_bfloat16* __restrict__ b_in, __nv_bfloat16* __restrict__ dst) {
  for (int o = threadIdx.x; o < width; o += blockDim.x) {
    const __nv_bfloat16* wr = W_in + static_cast<long>(o) * A;
    float acc = 0.f;
    for (int a = 0; a < A; a += 8) {
      uint4 raw = *reinterpret_cast<const uint4*>(wr + a);
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(w2[e]);
        acc = fmaf(f.x, xs[a + 2 * e], acc);
        acc = fmaf(f.y, xs[a + 2 * e + 1], acc);
      }
    }
    dst[o] = __float2bfloat16_rn(acc + (b_in ? __bfloat162float(b_in[o]) : 0.f));
  }
}

struct IoParams {
  int B, S, S_total, A, width, h_row_offset;
  const __nv_bfloat16* h;
  const float* a1;
  const float* a2;
  const float* b2;
  long ab_stride;
  float eps;
  const __nv_bfloat16* w_out;
  const __nv_bfloat16* b_out;
  float* x;
  float dt;
  const __nv_bfloat16* w_in;
  const __nv_bfloat16* b_in;
  __nv_bfloat16* h_next;
  int h_next_ld, h_next_rps, h_next_off;
};

__global__ void __launch_bounds__(256) action_in_kernel(const IoParams p) {
  __shared__ float xs[256];
  pdl_wait();
  const int b = blockIdx.x / p.S, s = blockIdx.x % p.S;
  for (int a = threadIdx.x; a < p.A; a += blockDim.x)
    xs[a] = bf16_round(p.x[(static_cast<long>(b) * p.S + s) * p.A + a]);
  __syncthreads();
  action_in_row(xs, p.A, p.width, p.w_in, p.b_in,
                p.h_next + (static_cast<long>(b) * p.h_next_rps + p.h_next_off + s) * p.h_next_ld);
  pdl_launch_dependents();
}

// Final norm -> action_out_proj -> Euler update -> next step's action_in_proj,
// all per action token (tokens are independent in these three ops).
__global__ void __launch_bounds__(256) euler_tail_kernel(const IoParams p) {
  extern __shared__ float ysh[];  // [width] normalized row, then [A] velocity / new x
  __shared__ float red[8];
  __shared__ float xs[256];
  pdl_wait();
  const int b = blockIdx.x / p.S, s = blockIdx.x % p.S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __nv_bfloat16* hr = p.h + (static_cast<long>(b) * p.S_total + p.h_row_offset + s) * p.width;
  float ss = 0.f;
  for (int k = threadIdx.x * 8; k < p.width; k += blockDim.x * 8) {
    uint4 raw = *reinterpret_cast<const uint4*>(hr + k);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __bfloat1622float2(h2[e]);
      ysh[k + 2 * e] = f.x;
      ysh[k + 2 * e + 1] = f.y;
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) tot += red[w];
  const float rstd = rsqrtf(tot / static_cast<float>(p.width) + p.eps);
  for (int k = threadIdx.x; k < p.width; k += blockDim.x) {
    float v = __fmul_rn(__fmul_rn(ysh[k], rstd), p.a1[k]);
    if (p.a2) v = __fmul_rn(v, p.a2[b * p.ab_stride + k]);
    if (p.b2) v = __fadd_rn(v, p.b2[b * p.ab_stride + k]);
    ysh[k] = bf16_round(v);
  }
  __syncthreads();
  // velocity v[a] = bf16(y · W_out[a] + b_out[a]); x += fp32(bf16(dt * v))
  for (int a = warp; a < p.A; a += blockDim.x >> 5) {
    const __nv_bfloat16* wr = p.w_out + static_cast<long>(a) * p.width;
    float acc = 0.f;
    for (int k = lane * 8; k < p.width; k += 256) {
      uint4 raw = *reinterpret_cast<const uint4*>(wr + k);
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(w2[e]);
        acc = fmaf(f.x, ysh[k + 2 * e], acc);
        acc = fmaf(f.y, ysh[k + 2 * e + 1], acc);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      const float v = bf16_round(acc + (p.b_out ? __bfloat162float(p.b_out[a]) : 0.f));
      float* xp = p.x + (static_cast<long>(b) * p.S + s) * p.A + a;
      const float xn = __fadd_rn(*xp, bf16_round(__fmul_rn(p.dt, v)));
      *xp = xn;
      xs[a] = bf16_round(xn);
    }
  }
  if (p.h_next) {
    __syncthreads();
    action_in_row(xs, p.A, p.width, p.w_in, p.b_in,
                  p.h_next + (static_cast<long>(b) * p.h_next_rps + p.h_next_off + s) * p.h_next_ld);
  }
  pdl_launch_dependents();
}

// y[t][k] = bf16(((x[t][k] * rstd[t]) * a1[k]) * a2[b][k] + b2[b][k]),
// rstd[t] = rsqrt(mean_k x[t][k]^2 + eps): the (Ada)RMSNorm of
// reflex/policies/pi05/modeling_pi05.py:73-99 in fp32 with one rounding to
// bf16, one CTA per token row.
struct NormParams {
  const __nv_bfloat16* x;
  int ldx, T, K, S;
  const float* a1;
  const float* a2;
  const float* b2;
  long ab_stride;
  float eps;
  __nv_bfloat16* y;
  int ldy;
};

__global__ void __launch_bounds__(128) rmsnorm_kernel(const NormParams p) {
  constexpr int kMaxChunks = 4;  // K <= 4096
  __shared__ float red[4];
  pdl_wait();
  // the next kernel may start its set-up (barriers, TMEM, weight prefetch)
  // now; its griddepcontrol.wait still waits for all of this grid
  pdl_launch_dependents();
  const int t = blockIdx.x;
  const int b = t / p.S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint4 raw[kMaxChunks];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int k = (c * 128 + threadIdx.x) * 8;
    if (k < p.K) raw[c] = *reinterpret_cast<const uint4*>(p.x + static_cast<long>(t) * p.ldx + k);
  }
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int k = (c * 128 + threadIdx.x) * 8;
    if (k >= p.K) continue;
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[c]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h2[e]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  const float rstd = rsqrtf((red[0] + red[1] + red[2] + red[3]) / static_cast<float>(p.K) + p.eps);
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int k = (c * 128 + threadIdx.x) * 8;
    if (k >= p.K) continue;
    const __nv_bfloat16* xv = reinterpret_cast<const __nv_bfloat16*>(&raw[c]);
    float a1[8], a2[8], b2[8];
    *reinterpret_cast<float4*>(a1) = *reinterpret_cast<const float4*>(p.a1 + k);
    *reinterpret_cast<float4*>(a1 + 4) = *reinterpret_cast<const float4*>(p.a1 + k + 4);
    const long bo = static_cast<long>(b) * p.ab_stride + k;
    if (p.a2) {
      *reinterpret_cast<float4*>(a2) = *reinterpret_cast<const float4*>(p.a2 + bo);
      *reinterpret_cast<float4*>(a2 + 4) = *reinterpret_cast<const float4*>(p.a2 + bo + 4);
    }
    if (p.b2) {
      *reinterpret_cast<float4*>(b2) = *reinterpret_cast<const float4*>(p.b2 + bo);
      *reinterpret_cast<float4*>(b2 + 4) = *reinterpret_cast<const float4*>(p.b2 + bo + 4);
    }
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float v = __fmul_rn(__fmul_rn(__bfloat162float(xv[e]), rstd), a1[e]);
      if (p.a2) v = __fmul_rn(v, a2[e]);
      if (p.b2) v = __fadd_rn(v, b2[e]);
      y[e] = v;
    }
    *reinterpret_cast<uint4*>(p.y + static_cast<long>(t) * p.ldy + k) =
        make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
  }
}

struct CopyRowsParams {
  __nv_bfloat16* dst;
  long dst_ld;
  int rpg, off, group;
  const __nv_bfloat16* src;
  long src_ld;
  int rows, width;
};

__global__ void __launch_bounds__(256) copy_rows_kernel(const CopyRowsParams p) {
  pdl_wait();
  const int chunks = p.width / 8;
  const long total = static_cast<long>(p.rows) * chunks;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / chunks), c = static_cast<int>(i % chunks);
    const long drow = static_cast<long>(r / p.group) * p.rpg + p.off + r % p.group;
    *reinterpret_cast<uint4*>(p.dst + drow * p.dst_ld + c * 8) =
        *reinterpret_cast<const uint4*>(p.src + r * p.src_ld + c * 8);
  }
  pdl_launch_dependents();
}

IoParams io_params(const rfx_action_io_desc& d) {
  IoParams p{};
  p.B = d.B;
  p.S = d.S;
  p.S_total = d.S_total;
  p.A = d.action_dim;
  p.width = d.width;
  p.h_row_offset = d.h_row_offset;
  p.h = static_cast<const __nv_bfloat16*>(d.h);
  p.a1 = d.norm_a1;
  p.a2 = d.norm_a2;
  p.b2 = d.norm_b2;
  p.ab_stride = d.norm_ab_stride;
  p.eps = d.eps;
  p.w_out = static_cast<const __nv_bfloat16*>(d.w_out);
  p.b_out = static_cast<const __nv_bfloat16*>(d.b_out);
  p.x = d.x;
  p.dt = d.dt;
  p.w_in = static_cast<const __nv_bfloat16*>(d.w_in);
  p.b_in = static_cast<const __nv_bfloat16*>(d.b_in);
  p.h_next = static_cast<__nv_bfloat16*>(d.h_next);
  p.h_next_ld = d.h_next_ld;
  p.h_next_rps = d.h_next_rows_per_stream;
  p.h_next_off = d.h_next_row_offset;
  return p;
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int validate_io(const rfx_action_io_desc& d, bool tail) {
  if (d.B < 1 || d.S < 1 || d.action_dim < 8 || d.action_dim % 8 || d.action_dim > 256 || d.width < 256 ||
      d.width % 256 || !d.x)
    return set_error(RFX_E_INVAL, "action io: need B,S>=1, action_dim%%8==0 (<=256), width%%256==0");
  if (tail) {
    if (!d.h || !d.w_out || !d.norm_a1 || d.S_total < d.S || d.h_row_offset < 0 ||
        d.h_row_offset + d.S > d.S_total || !a16(d.h) || !a16(d.w_out))
      return set_error(RFX_E_INVAL, "rfx_euler_tail: h/w_out/norm_a1 and row layout");
  }
  if (d.h_next || !tail) {
    if (!d.h_next || !d.w_in || !a16(d.w_in) || d.h_next_ld < d.width || d.h_next_rows_per_stream < d.S ||
        d.h_next_row_offset < 0 || d.h_next_row_offset + d.S > d.h_next_rows_per_stream)
      return set_error(RFX_E_INVAL, "action in-proj: h_next/w_in layout");
  }
  return RFX_OK;
}

int validate_time_cond(const rfx_time_cond_desc& d) {
  const bool embed_only = d.w_in == nullptr;
  if (d.n_t < 1 || d.n_t > kMaxRows || d.width < 256 || d.width % 256 || !d.t || !d.cond ||
      !a16(d.cond) || (!embed_only && (!d.w_out || !d.hidden || !a16(d.w_in) || !a16(d.w_out) || !a16(d.hidden))))
    return set_error(RFX_E_INVAL, "rfx_time_cond: need 1<=n_t<=16, width%%256==0, aligned weights");
  if (!(d.min_period > 0.0) || !(d.max_period > 0.0)) return set_error(RFX_E_INVAL, "rfx_time_cond: periods");
  if (!embed_only && static_cast<size_t>(d.n_t) * d.width * sizeof(float) > 200 * 1024)
    return set_error(RFX_E_UNSUPPORTED, "rfx_time_cond: n_t*width too large");
  return RFX_OK;
}

int launch_time_cond(const rfx_time_cond_desc& d, cudaStream_t stream, bool pdl) {
  const bool embed_only = d.w_in == nullptr;
  int rc0 = validate_time_cond(d);
  if (rc0) return rc0;
  __nv_bfloat16* emb = static_cast<__nv_bfloat16*>(d.cond);  // the embedding is staged in `cond`
  const int half = d.width / 2;
  const float* t = d.t;
  int n_t = d.n_t, width = d.width;
  double minp = d.min_period, maxp = d.max_period;
  int rc = launch_kernel(reinterpret_cast<const void*>(sinusoid_kernel), dim3((n_t * half + 255) / 256), dim3(256), 0,
                         stream, pdl, 1, t, n_t, width, minp, maxp, emb);
  if (rc || embed_only) return rc;
  const size_t smem = static_cast<size_t>(n_t) * width * sizeof(float);
  const void* gemv = reinterpret_cast<const void*>(gemv_bf16_silu_kernel);
  rc = ensure_smem_attr(gemv, 200 * 1024);
  if (rc) return rc;
  const __nv_bfloat16* in0 = emb;
  const __nv_bfloat16* w_in = static_cast<const __nv_bfloat16*>(d.w_in);
  const __nv_bfloat16* b_in = static_cast<const __nv_bfloat16*>(d.b_in);
  __nv_bfloat16* hid = static_cast<__nv_bfloat16*>(d.hidden);
  int n_out = width;
  dim3 grid((width + 7) / 8);
  rc = launch_kernel(gemv, grid, dim3(256), smem, stream, pdl, 1, in0, n_t, width, w_in, b_in, n_out, hid);
  if (rc) return rc;
  const __nv_bfloat16* in1 = hid;
  const __nv_bfloat16* w_out = static_cast<const __nv_bfloat16*>(d.w_out);
  const __nv_bfloat16* b_out = static_cast<const __nv_bfloat16*>(d.b_out);
  __nv_bfloat16* cond = static_cast<__nv_bfloat16*>(d.cond);
  return launch_kernel(gemv, grid, dim3(256), smem, stream, pdl, 1, in1, n_t, width, w_out, b_out, n_out, cond);
}

// conditioning rows padded to the next instantiated count
static int modulation_rows(int n_rows) { return n_rows <= 4 ? 4 : n_rows <= 8 ? 8 : n_rows <= 10 ? 10 : 16; }

int validate_modulation(const rfx_modulation_desc& d) {
  const int out = d.mode == RFX_ADARMS_SSG ? 3 * d.width : d.width;
  if ((d.mode != RFX_ADARMS_GATE && d.mode != RFX_ADARMS_SSG) || d.n_rows < 1 || d.n_rows > kMaxRows ||
      d.n_norms < 1 || d.width < 128 || d.width % 128 || !d.w || !d.b || !d.cond || !d.a2 || !d.gate ||
      (d.mode == RFX_ADARMS_SSG && !d.b2) || !a16(d.w) || !a16(d.cond) || !a16(d.a2) || !a16(d.gate) ||
      (d.b2 && !a16(d.b2)))
    return set_error(RFX_E_INVAL, "rfx_modulation: bad descriptor");
  if (static_cast<long>(d.n_norms) * out > (1L << 30))
    return set_error(RFX_E_UNSUPPORTED, "rfx_modulation: too many output rows");
  if (static_cast<size_t>(modulation_rows(d.n_rows)) * d.width * sizeof(float) > 100 * 1024)
    return set_error(RFX_E_UNSUPPORTED, "rfx_modulation: n_rows*width too large");
  return RFX_OK;
}

int launch_modulation(const rfx_modulation_desc& d, cudaStream_t stream, bool pdl) {
  int rc = validate_modulation(d);
  if (rc) return rc;
  const int out = d.mode == RFX_ADARMS_SSG ? 3 * d.width : d.width;
  const long rows = static_cast<long>(d.n_norms) * out;
  const int kr = modulation_rows(d.n_rows);
  const void* fn = kr == 4   ? reinterpret_cast<const void*>(modulation_kernel<4>)
                   : kr == 8 ? reinterpret_cast<const void*>(modulation_kernel<8>)
                   : kr == 10 ? reinterpret_cast<const void*>(modulation_kernel<10>)
                              : reinterpret_cast<const void*>(modulation_kernel<16>);
  const size_t smem = static_cast<size_t>(kr) * d.width * sizeof(float);
  rc = ensure_smem_attr(fn, 100 * 1024);
  if (rc) return rc;
  int nsm = 148;
  rfx_num_sms(&nsm);
  // one wave at two resident blocks per SM; each warp takes 4 rows per iteration
  dim3 grid(static_cast<unsigned>(std::min<long>((rows + 31) / 32, 2L * nsm)));
  const float* w = d.w;
  const float* bias = d.b;
  const __nv_bfloat16* cond = static_cast<const __nv_bfloat16*>(d.cond);
  int n_rows = d.n_rows, width = d.width, n_norms = d.n_norms, opn = out, mode = d.mode;
  float* a2 = d.a2;
  float* b2 = d.b2;
  float* gate = d.gate;
  return launch_kernel(fn, grid, dim3(256), smem, stream, pdl, 1, w, bias, cond, n_rows, width, n_norms, opn, mode, a2,
                       b2, gate);
}

int launch_action_in(const rfx_action_io_desc& d, cudaStream_t stream, bool pdl) {
  int rc = validate_io(d, false);
  if (rc) return rc;
  IoParams p = io_params(d);
  return launch_kernel(reinterpret_cast<const void*>(action_in_kernel), dim3(d.B * d.S), dim3(256), 0, stream, pdl, 1,
                       p);
}

int launch_euler_tail(const rfx_action_io_desc& d, cudaStream_t stream, bool pdl) {
  int rc = validate_io(d, true);
  if (rc) return rc;
  IoParams p = io_params(d);
  const size_t smem = static_cast<size_t>(d.width) * sizeof(float);
  const void* fn = reinterpret_cast<const void*>(euler_tail_kernel);
  rc = ensure_smem_attr(fn, static_cast<int>(smem > 48 * 1024 ? smem : 48 * 1024));
  if (rc) return rc;
  return launch_kernel(fn, dim3(d.B * d.S), dim3(256), smem, stream, pdl, 1, p);
}

int validate_rms_norm(const rfx_norm_desc& d) {
  if (d.T < 1 || d.K < 8 || d.K % 8 || d.K > 4096 || d.tokens_per_batch < 1 || !d.x || !d.y || !d.norm_a1 ||
      d.ldx < d.K || d.ldx % 8 || d.ldy < d.K || d.ldy % 8 || !a16(d.x) || !a16(d.y) || !a16(d.norm_a1) ||
      (d.norm_a2 && !a16(d.norm_a2)) || (d.norm_b2 && !a16(d.norm_b2)) || d.norm_ab_stride % 4)
    return set_error(RFX_E_INVAL, "rfx_rms_norm: need K%%8==0 (<=4096), 16-byte aligned rows and vectors");
  return RFX_OK;
}

int launch_rms_norm(const rfx_norm_desc& d, cudaStream_t stream, bool pdl) {
  int rc = validate_rms_norm(d);
  if (rc) return rc;
  NormParams p{static_cast<const __nv_bfloat16*>(d.x), d.ldx, d.T, d.K, d.tokens_per_batch, d.norm_a1, d.norm_a2,
               d.norm_b2, d.norm_ab_stride, d.eps, static_cast<__nv_bfloat16*>(d.y), d.ldy};
  return launch_kernel(reinterpret_cast<const void*>(rmsnorm_kernel), dim3(d.T), dim3(128), 0, stream, pdl, 1, p);
}

int validate_copy_rows(const rfx_copy_rows_desc& d) {
  if (!d.dst || !d.src || d.rows < 0 || d.width < 8 || d.width % 8 || d.group < 1 || d.dst_rows_per_group < 1 ||
      d.dst_row_offset < 0 || d.dst_row_offset + d.group > d.dst_rows_per_group || d.dst_ld < d.width ||
      d.dst_ld % 8 || d.src_ld < 0 || d.src_ld % 8 || (d.src_ld > 0 && d.src_ld < d.width) || !a16(d.dst) ||
      !a16(d.src))
    return set_error(RFX_E_INVAL, "rfx_copy_rows: bad layout (16-byte aligned rows of width%%8==0 required)");
  return RFX_OK;
}

int launch_copy_rows(const rfx_copy_rows_desc& d, cudaStream_t stream, bool pdl) {
  int rc = validate_copy_rows(d);
  if (rc || d.rows == 0) return rc;
  CopyRowsParams p{static_cast<__nv_bfloat16*>(d.dst), d.dst_ld, d.dst_rows_per_group, d.dst_row_offset, d.group,
                   static_cast<const __nv_bfloat16*>(d.src), d.src_ld, d.rows, d.width};
  const long total = static_cast<long>(d.rows) * (d.width / 8);
  const unsigned blocks = static_cast<unsigned>(std::min<long>((total + 255) / 256, 1184));
  return launch_kernel(reinterpret_cast<const void*>(copy_rows_kernel), dim3(blocks), dim3(256), 0, stream, pdl, 1,
                       p);
}

}  // namespace rfx

extern "C" int rfx_rms_norm(const rfx_norm_desc* d, void* stream) {
  if (!d) return rfx::set_error(RFX_E_INVAL, "rfx_rms_norm: null descriptor");
  return rfx::launch_rms_norm(*d, static_cast<cudaStream_t>(stream), rfx::pdl_enabled());
}

extern "C" int rfx_copy_rows(const rfx_copy_rows_desc* d, void* stream) {
  if (!d) return rfx::set_error(RFX_E_INVAL, "rfx_copy_rows: null descriptor");
  return rfx::launch_copy_rows(*d, static_cast<cudaStream_t>(stream), rfx::pdl_enabled());
}

extern "C" int rfx_time_cond(const rfx_time_cond_desc* d, void* stream) {
  if (!d) return rfx::set_error(RFX_E_INVAL, "rfx_time_cond: null descriptor");
  return rfx::launch_time_cond(*d, static_cast<cudaStream_t>(stream), rfx::pdl_enabled());
}
extern "C" int rfx_modulation(const rfx_modulation_desc* d, void* stream) {
  if (!d) return rfx::set_error(RFX_E_INVAL, "rfx_modulation: null descriptor");
  return rfx::launch_modulation(*d, static_cast<cudaStream_t>(stream), rfx::pdl_enabled());
}
extern "C" int rfx_action_in(const rfx_action_io_desc* d, void* stream) {
  if (!d) return rfx::set_error(RFX_E_INVAL, "rfx_action_in: null descriptor");
  return rfx::launch_action_in(*d, static_cast<cudaStream_t>(stream), rfx::pdl_enabled());
}
extern "C" int rfx_euler_tail(const rfx_action_io_desc* d, void* stream) {
  if (!d) return rfx::set_error(RFX_E_INVAL, "rfx_euler_tail: null descriptor");
  return rfx::launch_euler_tail(*d, static_cast<cudaStream_t>(stream), rfx::pdl_enabled());
}
