// Similarity gate of the observation-embedding cache: decides on the device
// whether a camera image is close enough to the last one that was embedded
// for its embedding to be reused, without reading the image back to the host.
//
//   RFX_EMBED_CACHE_POOL_MSE: PI05PrefixEmbedder.forward's check
//     (reflex/policies/pi05/modeling_pi05.py:173-247): adaptive 2-D average
//     pooling of every channel to P x P (P = 32; cell (i, j) averages rows
//     [floor(i H / P), ceil((i + 1) H / P)) and the same for columns), then
//     the mean squared difference per image against the stored features; a
//     hit needs mse < threshold for every image of the batch.
//   RFX_EMBED_CACHE_BILINEAR_COS: LastFrameCache.get_or_compute
//     (reflex/optimizations/dynamic_embedding_cache.py:284-392): bilinear
//     resampling to P x P (P = 16, half-pixel centres, source coordinate
//     clamped at 0: F.interpolate(..., align_corners=False)), flattened per
//     image, cosine similarity x.y / (max(|x|, 1e-12) max(|y|, 1e-12)) per
//     image, averaged over the batch; a hit needs mean >= threshold.
//
// Two launches: features + per-image sums (one CTA per image, channels in
// order, fixed-order block reductions: deterministic), then the decision (one
// CTA), which on a miss (or with no stored features) copies the new features
// into the store, as the reference updates its cache only when it embeds.
#include "rfx_internal.h"

namespace rfx {
namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ float load_px(const void* img, long i, bool bf16) {
  return bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(img)[i]) : static_cast<const float*>(img)[i];
}

// Fixed-order sum over the block: warp trees, then warp 0 over the warp sums.
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
  if (w == 0) t = warp_sum(t);
  return t;  // valid in thread 0
}

__global__ void __launch_bounds__(kThreads) embed_features_kernel(rfx_embed_cache_desc d) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int P = d.pool, t = threadIdx.x;
  const bool active = t < P * P;
  const int py = active ? t / P : 0, px = active ? t % P : 0;
  const bool bf16 = d.in_dtype == RFX_DTYPE_BF16;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f;
  for (int c = 0; c < d.C; ++c) {
    const long plane = (static_cast<long>(b) * d.C + c) * d.H * d.W;
    float f = 0.f;
    if (active) {
      if (d.mode == RFX_EMBED_CACHE_POOL_MSE) {
        const int y0 = (py * d.H) / P, y1 = ((py + 1) * d.H + P - 1) / P;
        const int x0 = (px * d.W) / P, x1 = ((px + 1) * d.W + P - 1) / P;
        float acc = 0.f;
        for (int y = y0; y < y1; ++y)
          for (int x = x0; x < x1; ++x) acc += load_px(d.image, plane + static_cast<long>(y) * d.W + x, bf16);
        f = acc / static_cast<float>((y1 - y0) * (x1 - x0));
      } else {
        const float sy = static_cast<float>(d.H) / P, sx = static_cast<float>(d.W) / P;
        const float fy = fmaxf(sy * (py + 0.5f) - 0.5f, 0.f), fx = fmaxf(sx * (px + 0.5f) - 0.5f, 0.f);
        const int y0 = min(static_cast<int>(fy), d.H - 1), x0 = min(static_cast<int>(fx), d.W - 1);
        const int y1 = min(y0 + 1, d.H - 1), x1 = min(x0 + 1, d.W - 1);
        const float ly = fy - y0, lx = fx - x0;
        const float v00 = load_px(d.image, plane + static_cast<long>(y0) * d.W + x0, bf16);
        const float v01 = load_px(d.image, plane + static_cast<long>(y0) * d.W + x1, bf16);
        const float v10 = load_px(d.image, plane + static_cast<long>(y1) * d.W + x0, bf16);
        const float v11 = load_px(d.image, plane + static_cast<long>(y1) * d.W + x1, bf16);
        f = (1.f - ly) * ((1.f - lx) * v00 + lx * v01) + ly * ((1.f - lx) * v10 + lx * v11);
      }
      const long fi = (static_cast<long>(b) * d.C + c) * P * P + t;
      d.feat_new[fi] = f;
      const float p = d.feat_prev[fi];
      if (d.mode == RFX_EMBED_CACHE_POOL_MSE) {
        s0 = fmaf(f - p, f - p, s0);
      } else {
        s0 = fmaf(f, p, s0);
        s1 = fmaf(f, f, s1);
        s2 = fmaf(p, p, s2);
      }
    }
  }
  s0 = block_sum(s0, red);
  if (d.mode != RFX_EMBED_CACHE_POOL_MSE) {
    s1 = block_sum(s1, red);
    s2 = block_sum(s2, red);
  }
  if (t == 0) {
    d.sums[3 * b + 0] = s0;
    d.sums[3 * b + 1] = s1;
    d.sums[3 * b + 2] = s2;
  }
}

__global__ void __launch_bounds__(kThreads) embed_decide_kernel(rfx_embed_cache_desc d) {
  __shared__ int hit_s;
  if (threadIdx.x == 0) {
    bool hit = d.state[0] != 0;
    float mean = 0.f;
    for (int b = 0; b < d.B; ++b) {
      const float* s = d.sums + 3 * b;
      if (d.mode == RFX_EMBED_CACHE_POOL_MSE) {
        const float mse = s[0] / static_cast<float>(d.C * d.pool * d.pool);
        d.metric[b] = mse;
        hit = hit && mse < d.threshold;
      } else {
        const float sim = s[0] / (fmaxf(sqrtf(s[1]), 1e-12f) * fmaxf(sqrtf(s[2]), 1e-12f));
        d.metric[b] = sim;
        mean += sim;
      }
    }
    if (d.mode != RFX_EMBED_CACHE_POOL_MSE) hit = hit && mean / static_cast<float>(d.B) >= d.threshold;
    hit_s = hit ? 1 : 0;
    d.state[1] = hit_s;
    if (!hit) d.state[0] = 1;  // the store holds features from now on
  }
  __syncthreads();
  if (!hit_s) {
    const long n = static_cast<long>(d.B) * d.C * d.pool * d.pool;
    for (long i = threadIdx.x; i < n; i += blockDim.x) d.feat_prev[i] = d.feat_new[i];
  }
}

}  // namespace
}  // namespace rfx

extern "C" int rfx_embed_cache_check(const rfx_embed_cache_desc* desc, void* stream) {
  using namespace rfx;
  if (!desc) return set_error(RFX_E_INVAL, "rfx_embed_cache_check: null descriptor");
  const rfx_embed_cache_desc& d = *desc;
  if (d.mode != RFX_EMBED_CACHE_POOL_MSE && d.mode != RFX_EMBED_CACHE_BILINEAR_COS)
    return set_error(RFX_E_INVAL, "rfx_embed_cache_check: mode");
  if (d.B < 1 || d.C < 1 || d.H < 1 || d.W < 1 || d.pool < 1 || d.pool * d.pool > kThreads)
    return set_error(RFX_E_INVAL, "rfx_embed_cache_check: need B, C, H, W >= 1 and pool * pool <= %d", kThreads);
  if (d.mode == RFX_EMBED_CACHE_POOL_MSE && (d.H < d.pool || d.W < d.pool))
    return set_error(RFX_E_INVAL, "rfx_embed_cache_check: adaptive pooling needs H, W >= pool");
  if (d.in_dtype != RFX_DTYPE_F32 && d.in_dtype != RFX_DTYPE_BF16)
    return set_error(RFX_E_INVAL, "rfx_embed_cache_check: image dtype must be fp32 or bf16");
  if (!d.image || !d.feat_prev || !d.feat_new || !d.sums || !d.state || !d.metric)
    return set_error(RFX_E_INVAL, "rfx_embed_cache_check: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rfx_embed_cache_desc a = d;
  int rc = launch_kernel(reinterpret_cast<const void*>(embed_features_kernel), dim3(d.B), dim3(kThreads), 0, st,
                         false, 1, a);
  if (rc) return rc;
  return launch_kernel(reinterpret_cast<const void*>(embed_decide_kernel), dim3(1), dim3(kThreads), 0, st, false, 1,
                       a);
}
