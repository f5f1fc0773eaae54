// The SigLIP vision tower's own kernels: patch extraction, LayerNorm and the
// per-image multi-head attention.  The projections (q/k/v, out, fc1 + GELU,
// fc2, the patch convolution as a GEMM and the PaliGemma projector) run on
// rfx_linear.  Replaces the transformers SiglipVisionModel that the reference
// reaches through the VLM's image embedder
// (reflex/policies/pi05/modeling_pi05.py:141-158, :244).
#include "rfx_internal.h"

namespace rfx {
namespace {

// ------------------------------------------------------------ patches ----
struct PatchParams {
  const float* image;
  __nv_bfloat16* out;
  int B, C, H, W, P, G, ldo, kp;  // kp = C * P * P
};

// One thread per pair of output columns of one patch row.
__global__ void __launch_bounds__(256) patches_kernel(const PatchParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int pairs = p.ldo / 2;
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long total = static_cast<long>(p.B) * p.G * p.G * pairs;
  if (idx >= total) return;
  const int c2 = static_cast<int>(idx % pairs);
  const long t = idx / pairs;
  const int gx = static_cast<int>(t % p.G);
  const int gy = static_cast<int>((t / p.G) % p.G);
  const int b = static_cast<int>(t / (static_cast<long>(p.G) * p.G));
  float v[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int k = 2 * c2 + e;
    v[e] = 0.f;
    if (k < p.kp) {
      const int c = k / (p.P * p.P), r = k - c * p.P * p.P;
      const int py = r / p.P, px = r - py * p.P;
      v[e] = p.image[((static_cast<long>(b) * p.C + c) * p.H + gy * p.P + py) * p.W + gx * p.P + px];
    }
  }
  *reinterpret_cast<uint32_t*>(p.out + t * p.ldo + 2 * c2) = pack_bf16x2(v[0], v[1]);
}

// ---------------------------------------------------------- LayerNorm ----
struct LnParams {
  const __nv_bfloat16* x;
  int ldx;
  const float* w;
  const float* b;
  float eps;
  __nv_bfloat16* y;
  int ldy, T, C;
};

// One warp per row; lane j takes the row's 16-byte chunks j, j + 32, ...
// (C % 8 == 0, C <= 2048: at most eight chunks a lane), all loaded at once and
// kept in registers for the mean, the variance and the output.
constexpr int kLnChunks = 8;
__global__ void __launch_bounds__(256) layernorm_kernel(const LnParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= p.T) return;
  const int nch = p.C / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(p.x + static_cast<long>(t) * p.ldx);
  float v[kLnChunks][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kLnChunks; ++i) {
    const int c = i * 32 + lane;
    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    if (c < nch) raw = xr[c];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      v[i][2 * e] = f.x;
      v[i][2 * e + 1] = f.y;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) s += v[i][e];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(p.C);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kLnChunks; ++i) {
    if (i * 32 + lane >= nch) continue;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float a = v[i][e] - mean;
      q += a * a;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q / static_cast<float>(p.C) + p.eps);
  uint4* yr = reinterpret_cast<uint4*>(p.y + static_cast<long>(t) * p.ldy);
#pragma unroll
  for (int i = 0; i < kLnChunks; ++i) {
    const int c = i * 32 + lane;
    if (c >= nch) continue;
    const float4 w0 = *reinterpret_cast<const float4*>(p.w + 8 * c);
    const float4 w1 = *reinterpret_cast<const float4*>(p.w + 8 * c + 4);
    const float4 b0 = *reinterpret_cast<const float4*>(p.b + 8 * c);
    const float4 b1 = *reinterpret_cast<const float4*>(p.b + 8 * c + 4);
    const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    uint4 o;
    o.x = pack_bf16x2((v[i][0] - mean) * rstd * w[0] + b[0], (v[i][1] - mean) * rstd * w[1] + b[1]);
    o.y = pack_bf16x2((v[i][2] - mean) * rstd * w[2] + b[2], (v[i][3] - mean) * rstd * w[3] + b[3]);
    o.z = pack_bf16x2((v[i][4] - mean) * rstd * w[4] + b[4], (v[i][5] - mean) * rstd * w[5] + b[5]);
    o.w = pack_bf16x2((v[i][6] - mean) * rstd * w[6] + b[6], (v[i][7] - mean) * rstd * w[7] + b[7]);
    yr[c] = o;
  }
}

// ------------------------------------------------------ ViT attention ----
// One CTA per (128 query rows, head, image); all N <= 256 keys of the image
// in one pass.  Q, K and V are staged by every thread from the q/k/v
// projection rows into shared memory, zero-padded to 128 dims:
//   Q, K: K-major SW128 tiles (dim atoms of 64), V: MN-major SW128 tiles
//   (64-key groups x dim atoms of 64).
// S = Q K^T (M 128, N 256, D/16 k-steps) goes to TMEM columns 256..511; eight
// worker warps (two per TMEM lane quadrant, each on 128 keys) take the row
// maximum, then write P = 2^(s*scale*log2e - m) as bf16 pairs over the first
// half of their own S columns; O = P V (A from TMEM, N = D rounded up to 64)
// accumulates in columns 0..127 and is divided by the row sum on the way out.
constexpr int kVQ = 128;
constexpr int kVKeys = 256;
constexpr int kVOffQ = 0;         // 2 x [128 rows x 64 dims] bf16
constexpr int kVOffK = 32768;     // 2 x [256 keys x 64 dims] bf16
constexpr int kVOffV = 98304;     // 4 key groups x 2 x [64 keys x 64 dims] bf16
constexpr int kVOffBar = 163840;  // s_full, p_ready, o_full, TMEM address
constexpr int kVOffX = kVOffBar + 64;   // [2][128] row maxima, [2][128] row sums
constexpr int kVSmem = kVOffX + 2048 + 1024;
constexpr int kVThreads = 320;
static_assert(kVSmem <= 227 * 1024, "vit attention shared memory");

struct VitParams {
  const __nv_bfloat16* qkv;
  int ld_qkv;
  __nv_bfloat16* out;
  int ld_out;
  int N, H, D;
  float scale_log2;
  int* status;
};

// byte offset of 16-byte chunk `c` (0..7) of row `r` in a 128-byte-row SW128 tile
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

// Named barrier over the two worker warps of TMEM lane quadrant `quad` that
// ANDs a flag over them.
__device__ __forceinline__ bool vit_pair_all(int quad, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, 64, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u), "r"(2 + quad)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(kVThreads, 1) vit_attention_kernel(const VitParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kVOffBar);
  uint64_t* s_full = bars;
  uint64_t* p_ready = bars + 1;
  uint64_t* o_full = bars + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  float* mx_x = reinterpret_cast<float*>(smem + kVOffX);
  float* l_x = mx_x + 256;
  if (threadIdx.x == 0) {
    mbar_init(s_full, 1);
    mbar_init(p_ready, 8);
    mbar_init(o_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  pdl_wait();  // q/k/v come from the previous kernel
  const int dch = p.D / 8;  // 16-byte chunks of a row that hold data
  const long row0 = static_cast<long>(b) * p.N;
  const __nv_bfloat16* qsrc = p.qkv + static_cast<long>(h) * p.D;
  const __nv_bfloat16* ksrc = p.qkv + static_cast<long>(p.H + h) * p.D;
  const __nv_bfloat16* vsrc = p.qkv + static_cast<long>(2 * p.H + h) * p.D;
  // every 16-byte chunk of data by an asynchronous copy (all of a thread's
  // copies in flight at once), the padding chunks and rows by plain zero stores
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  for (int i = threadIdx.x; i < kVQ * 16; i += kVThreads) {
    const int r = i >> 4, c = i & 15;
    const int n = qt * kVQ + r;
    uint8_t* dst = smem + kVOffQ + (c >> 3) * 16384 + sw128_off(r, c & 7);
    if (n < p.N && c < dch)
      cp_async16(dst, qsrc + (row0 + n) * p.ld_qkv + c * 8);
    else
      *reinterpret_cast<uint4*>(dst) = zero;
  }
  for (int i = threadIdx.x; i < kVKeys * 16; i += kVThreads) {
    const int r = i >> 4, c = i & 15;
    uint8_t* kd = smem + kVOffK + (c >> 3) * 32768 + sw128_off(r, c & 7);
    uint8_t* vd = smem + kVOffV + (r >> 6) * 16384 + (c >> 3) * 8192 + sw128_off(r & 63, c & 7);
    if (r < p.N && c < dch) {
      cp_async16(kd, ksrc + (row0 + r) * p.ld_qkv + c * 8);
      cp_async16(vd, vsrc + (row0 + r) * p.ld_qkv + c * 8);
    } else {
      *reinterpret_cast<uint4*>(kd) = zero;
      *reinterpret_cast<uint4*>(vd) = zero;
    }
  }
  cp_async_commit();
  cp_async_wait_all();
  fence_proxy_async_smem();  // shared-memory writes -> tensor-core operand reads
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmO = tmem, tmS = tmem + 256;
  const int dq = (p.D + 15) / 16;  // k-steps of Q K^T
  const int dn = (p.D + 63) / 64 * 64;  // N of P V (whole dim atoms)
  if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_f16(kVQ, kVKeys, true);
      for (int ks = 0; ks < dq; ++ks) {
        const int a = ks >> 2, kk = ks & 3;
        const uint64_t ad = make_sdesc_sw128(smem_u32(smem + kVOffQ + a * 16384) + kk * 32, 16, 1024);
        const uint64_t bd = make_sdesc_sw128(smem_u32(smem + kVOffK + a * 32768) + kk * 32, 16, 1024);
        umma_f16_ss(tmS, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
      }
      umma_commit(s_full);
      if (mbar_wait(p_ready, 0, p.status, kDevTimeoutConvert)) {
        tc_fence_after();
        const uint32_t idesc_o = make_idesc_f16(kVQ, dn, true, true);
        for (int ks = 0; ks < kVKeys / 16; ++ks) {
          const int g = ks >> 2, kk = ks & 3;
          const uint64_t bd = make_sdesc_sw128(smem_u32(smem + kVOffV + g * 16384) + kk * 2048, 8192, 1024);
          const uint32_t pa = tmS + static_cast<uint32_t>(ks < 8 ? ks * 8 : 128 + (ks - 8) * 8);
          umma_f16_ts(tmO, pa, bd, idesc_o, ks > 0 ? 1u : 0u);
        }
      }
      umma_commit(o_full);  // arrives once every MMA issued above has completed
    }
  } else if (warp >= 2) {
    const int quad = warp & 3;
    const int ch = (warp - 2) >> 2;  // keys 128 ch .. 128 ch + 127
    const int r = quad * 32 + lane;  // query row in the tile == TMEM lane
    const uint32_t lb = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t sc = tmS + lb + static_cast<uint32_t>(ch * 128);
    bool ok = __all_sync(0xffffffffu, mbar_wait(s_full, 0, p.status, kDevTimeoutMmaDone));
    tc_fence_after();
    float mx = -INFINITY;
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t rr[16];
        tmem_ld16(sc + c * 16, rr);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (ch * 128 + c * 16 + e < p.N) mx = fmaxf(mx, __uint_as_float(rr[e]));
      }
    }
    mx_x[ch * 128 + r] = mx;
    ok = vit_pair_all(quad, ok);
    const float m = fmaxf(mx_x[r], mx_x[128 + r]);
    const float msub = m == -INFINITY ? 0.f : m * p.scale_log2;
    float l = 0.f;
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t rr[2][16];
        tmem_ld16(sc + c * 32, rr[0]);
        tmem_ld16(sc + c * 32 + 16, rr[1]);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const int key = ch * 128 + c * 32 + q * 16 + e;
            const float p0 = key < p.N ? bf16_round(ex2_approx(__uint_as_float(rr[q][e]) * p.scale_log2 - msub)) : 0.f;
            const float p1 =
                key + 1 < p.N ? bf16_round(ex2_approx(__uint_as_float(rr[q][e + 1]) * p.scale_log2 - msub)) : 0.f;
            l += p0 + p1;
            pk[q * 8 + e / 2] = pack_bf16x2(p0, p1);
          }
        tmem_st16(sc + c * 16, pk);  // over S columns already read
      }
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(p_ready);
    l_x[ch * 128 + r] = l;
    ok = vit_pair_all(quad, ok);
    // every issued MMA completes before TMEM is read or freed
    const bool done = __all_sync(0xffffffffu, mbar_wait(o_full, 0, p.status, kDevTimeoutMmaDone));
    tc_fence_after();
    const int n = qt * kVQ + r;
    const float lsum = l_x[r] + l_x[128 + r];
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    if (ok && done) {
#pragma unroll 1
      for (int c = ch; c < dq; c += 2) {  // 16 output dims per step, alternating between the pair
        uint32_t rr[16];
        tmem_ld16(tmO + lb + c * 16, rr);
        tmem_wait_ld();
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int d0 = c * 16 + j * 8;
            if (d0 >= p.D) break;
            uint4 o;
            o.x = pack_bf16x2(__uint_as_float(rr[8 * j + 0]) * inv, __uint_as_float(rr[8 * j + 1]) * inv);
            o.y = pack_bf16x2(__uint_as_float(rr[8 * j + 2]) * inv, __uint_as_float(rr[8 * j + 3]) * inv);
            o.z = pack_bf16x2(__uint_as_float(rr[8 * j + 4]) * inv, __uint_as_float(rr[8 * j + 5]) * inv);
            o.w = pack_bf16x2(__uint_as_float(rr[8 * j + 6]) * inv, __uint_as_float(rr[8 * j + 7]) * inv);
            *reinterpret_cast<uint4*>(p.out + (row0 + n) * p.ld_out + static_cast<long>(h) * p.D + d0) = o;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool a16v(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace

int validate_patches(const rfx_patches_desc& d) {
  if (d.B < 1 || d.C < 1 || d.patch < 1 || d.H != d.W || d.H % d.patch || !d.image || !d.out || !a16v(d.out) ||
      d.ldo % 64 || d.ldo < d.C * d.patch * d.patch)
    return set_error(RFX_E_INVAL, "rfx_patches: square image with H %% patch == 0, ldo %% 64 == 0 and >= C*P*P");
  return RFX_OK;
}

int launch_patches(const rfx_patches_desc& d, cudaStream_t stream, bool pdl) {
  int rc = validate_patches(d);
  if (rc) return rc;
  PatchParams p{d.image, static_cast<__nv_bfloat16*>(d.out), d.B, d.C, d.H, d.W, d.patch, d.H / d.patch, d.ldo,
                d.C * d.patch * d.patch};
  const long total = static_cast<long>(d.B) * p.G * p.G * (d.ldo / 2);
  return launch_kernel(reinterpret_cast<const void*>(patches_kernel), dim3(static_cast<unsigned>((total + 255) / 256)),
                       dim3(256), 0, stream, pdl, 1, p);
}

int validate_layer_norm(const rfx_layer_norm_desc& d) {
  if (d.T < 1 || d.C < 8 || d.C % 8 || d.C > 2048 || !d.x || !d.y || !d.w || !d.b || d.ldx < d.C || d.ldx % 8 ||
      d.ldy < d.C || d.ldy % 8 || !a16v(d.x) || !a16v(d.y) || !a16v(d.w) || !a16v(d.b))
    return set_error(RFX_E_INVAL, "rfx_layer_norm: need C %% 8 == 0 (<= 2048), 16-byte aligned rows and vectors");
  return RFX_OK;
}

int launch_layer_norm(const rfx_layer_norm_desc& d, cudaStream_t stream, bool pdl) {
  int rc = validate_layer_norm(d);
  if (rc) return rc;
  LnParams p{static_cast<const __nv_bfloat16*>(d.x), d.ldx, d.w, d.b, d.eps, static_cast<__nv_bfloat16*>(d.y),
             d.ldy, d.T, d.C};
  return launch_kernel(reinterpret_cast<const void*>(layernorm_kernel), dim3((d.T + 7) / 8), dim3(256), 0, stream,
                       pdl, 1, p);
}

int validate_vit_attention(const rfx_vit_attn_desc& d) {
  if (d.B < 1 || d.B > 65535 || d.N < 1 || d.N > kVKeys || d.H < 1 || d.H > 65535 || d.D < 8 || d.D > 128 ||
      d.D % 8 || !d.qkv || !d.out || !a16v(d.qkv) || !a16v(d.out) || d.ld_qkv % 8 || d.ld_qkv < 3 * d.H * d.D ||
      d.ld_out % 8 || d.ld_out < d.H * d.D)
    return set_error(RFX_E_INVAL,
                     "rfx_vit_attention: need N <= 256, D %% 8 == 0 (<= 128), 16-byte aligned rows of q|k|v");
  return RFX_OK;
}

int launch_vit_attention(const rfx_vit_attn_desc& d, cudaStream_t stream, bool pdl) {
  int rc = validate_vit_attention(d);
  if (rc) return rc;
  const void* fn = reinterpret_cast<const void*>(vit_attention_kernel);
  rc = ensure_smem_attr(fn, kVSmem);
  if (rc) return rc;
  VitParams p{static_cast<const __nv_bfloat16*>(d.qkv), d.ld_qkv, static_cast<__nv_bfloat16*>(d.out), d.ld_out,
              d.N, d.H, d.D, d.scale * 1.4426950408889634f, device_status_ptr()};
  return launch_kernel(fn, dim3((d.N + kVQ - 1) / kVQ, d.H, d.B), dim3(kVThreads), kVSmem, stream, pdl, 1, p);
}

}  // namespace rfx

extern "C" int rfx_patches(const rfx_patches_desc* d, void* stream) {
  if (!d) return rfx::set_error(RFX_E_INVAL, "rfx_patches: null descriptor");
  return rfx::launch_patches(*d, static_cast<cudaStream_t>(stream), rfx::pdl_enabled());
}
extern "C" int rfx_layer_norm(const rfx_layer_norm_desc* d, void* stream) {
  if (!d) return rfx::set_error(RFX_E_INVAL, "rfx_layer_norm: null descriptor");
  return rfx::launch_layer_norm(*d, static_cast<cudaStream_t>(stream), rfx::pdl_enabled());
}
extern "C" int rfx_vit_attention(const rfx_vit_attn_desc* d, void* stream) {
  if (!d) return rfx::set_error(RFX_E_INVAL, "rfx_vit_attention: null descriptor");
  return rfx::launch_vit_attention(*d, static_cast<cudaStream_t>(stream), rfx::pdl_enabled());
}
