// KV quantize-append into a ring buffer.
//
// Replaces the reference's per-(batch, head, token) quantizers:
//   * reflex/layers/streaming_attention.py:211-218  (StreamingAttention._quantize,
//     uint8 asymmetric min/max with zero-point, every op in the activation dtype)
//   * reflex/layers/quantize_kernel.py:6-79         (Triton _quantize_store_kernel,
//     same scheme, cache offset = l_offset + token)
// and adds the int8 symmetric per-token/per-head scheme (scale = absmax/127 in
// fp32, q = clamp(rne(x/scale), -127, 127)).
//
// Layout: one warp per four (b, h, token) rows of D = 256 elements; each lane
// owns 8 contiguous elements of a row (one 16-byte bf16 vector or two fp32
// vectors) and reductions are warp shuffles.  The destination slot of token l is
//   region_base + (region_off + l) % region_len
// so an append that wraps around the ring window is one launch, and eviction
// of the oldest frame is simply overwriting its slots (no data movement).
// Grid: x = blocks of 32 tokens, y = (b, h), z = {K, V}.
#include "rfx_internal.h"

namespace rfx {

namespace {

constexpr int kD = 256;
constexpr int kWarpsPerBlock = 8;

template <typename T>
struct Vec8 {
  float v[8];
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Rounds an fp32 intermediate to the activation dtype (identity for fp32).
template <typename T>
__device__ __forceinline__ float to_act(float x);
template <>
__device__ __forceinline__ float to_act<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_act<__nv_bfloat16>(float x) { return bf16_round(x); }

template <typename T>
__device__ __forceinline__ void store_act(T* p, float x);
template <>
__device__ __forceinline__ void store_act<float>(float* p, float x) { *p = x; }
template <>
__device__ __forceinline__ void store_act<__nv_bfloat16>(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }

struct QuantArgs {
  const void* x[2];      // K and V inputs, [B][H][L][D]
  long xs_b, xs_h, xs_l;  // element strides
  void* q[2];             // ring payload, [B][H][C][D] (int8 or uint8)
  long qs_b, qs_h, qs_c;
  void* scale[2];         // [B][H][C]: fp32 (i8 mode) or activation dtype (u8 mode)
  void* zp[2];            // [B][H][C] activation dtype (u8 mode only)
  long ss_b, ss_h, ss_c;
  int B, H, L;
  int region_base, region_off, region_len;
};

// Packed fp32x2 arithmetic (sm_100): two round-to-nearest fp32 operations per
// instruction, each lane exactly as the scalar one.
__device__ __forceinline__ unsigned long long pack_f32x2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float lo_f32(unsigned long long v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float hi_f32(unsigned long long v) {
  return __uint_as_float(static_cast<uint32_t>(v >> 32));
}
// max that returns NaN when either operand is NaN
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ unsigned long long mul_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long add_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long sub_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// int8 symmetric quantization of one lane's 8 values of a row, packed little
// endian into two words: q = clamp(rne(x / scale), -127, 127), exactly as with
// rintf(__fdiv_rn(x, scale)), but from a product with rcp = __frcp_rn(scale),
// the correctly rounded 1 / scale.
//
// Error bound: |x| <= absmax and scale = fl(absmax / 127) is a normal float,
// so the exact quotient q has |q| <= 127 (1 + 2^-23); then y = fl(x * rcp)
// and fl(q) both lie within |q| * (3 * 2^-24 + 2^-48) + 2^-149, under 2.3e-5,
// of q.  Hence |y| < 127.5 (rne(y) needs no clamp), and whenever y is at least
// 2^-14 (6.1e-5) away from every half-integer, fl(q) is on the same side of
// all of them and on none, so both round to the same integer.  Values closer
// than that (bf16 inputs put about 0.2 % of the quotients there, most on a
// tie) are divided in a second pass; a denormal scale divides all 8.
//
// Rounding: t = y + 1.5 * 2^23 holds rne(y) in its low mantissa bits, so the
// low byte of t's bit pattern is the two's-complement int8 and t - 1.5 * 2^23
// is rne(y) as a float; y - rne(y) is exact (Sterbenz).  A NaN input fails
// the distance test and takes the divide, as before.
__device__ __forceinline__ void quant8_i8(const float (&v)[8], float scale, float rcp, uint32_t (&packed)[2]) {
  constexpr float kMagic = 12582912.0f;     // 1.5 * 2^23
  constexpr float kFar = 0.5f - 0x1p-14f;   // |y - rne(y)| <= kFar: 2^-14 or more from a half-integer
  uint32_t tb[8];
  if (scale >= 0x1p-126f) {
    // two values per instruction (packed fp32x2, each lane rounded as the
    // scalar op); the largest distance to a rounded value decides the pass
    const unsigned long long r2 = pack_f32x2(rcp, rcp), m2 = pack_f32x2(kMagic, kMagic);
    float dmax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const unsigned long long y = mul_f32x2(pack_f32x2(v[i], v[i + 1]), r2);
      const unsigned long long t = add_f32x2(y, m2);
      const unsigned long long d = sub_f32x2(y, sub_f32x2(t, m2));
      dmax = max_nan(dmax, max_nan(fabsf(lo_f32(d)), fabsf(hi_f32(d))));
      tb[i] = __float_as_uint(lo_f32(t));
      tb[i + 1] = __float_as_uint(hi_f32(t));
    }
    // a NaN distance (NaN input) fails the test and takes the divide
    const bool near = !(dmax <= kFar);
    if (near) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float y = __fmul_rn(v[i], rcp);
        const float t = __uint_as_float(tb[i]);
        if (!(fabsf(__fsub_rn(y, __fsub_rn(t, kMagic))) <= kFar))
          tb[i] = __float_as_uint(__fadd_rn(fminf(fmaxf(rintf(__fdiv_rn(v[i], scale)), -127.f), 127.f), kMagic));
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float r = fminf(fmaxf(rintf(__fdiv_rn(v[i], scale)), -127.f), 127.f);
      tb[i] = __float_as_uint(__fadd_rn(r, kMagic));
    }
  }
  packed[0] = __byte_perm(__byte_perm(tb[0], tb[1], 0x0040), __byte_perm(tb[2], tb[3], 0x0040), 0x5410);
  packed[1] = __byte_perm(__byte_perm(tb[4], tb[5], 0x0040), __byte_perm(tb[6], tb[7], 0x0040), 0x5410);
}

// One warp quantizes kRowsPerWarp consecutive tokens of one (b, h): every
// row's 16-byte loads are issued first, and in the int8 scheme lane j computes
// row j's scale and reciprocal (one exact divide per row instead of one per
// lane), broadcast by shuffles.
constexpr int kRowsPerWarp = 4;

template <typename Tin, int MODE>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, 4) kv_quant_append_kernel(const QuantArgs a) {
  pdl_wait();
  // the next kernel may start its set-up now; its griddepcontrol.wait still
  // waits for all of this grid
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid: x = token blocks, y = b * H + h, z = {K, V}; each thread divides
  // twice (b, and the ring offset), never per row
  const int which = blockIdx.z;
  const int b = static_cast<int>(blockIdx.y) / a.H;
  const int h = static_cast<int>(blockIdx.y) - b * a.H;
  const int l0 = (static_cast<int>(blockIdx.x) * kWarpsPerBlock + warp) * kRowsPerWarp;
  if (l0 >= a.L) return;
  const int off = a.region_off % a.region_len;
  const Tin* src = static_cast<const Tin*>(a.x[which]) + b * a.xs_b + h * a.xs_h + lane * 8;
  uint8_t* qbase = static_cast<uint8_t*>(a.q[which]) + b * a.qs_b + h * a.qs_h + lane * 8;
  const long sbase = b * a.ss_b + h * a.ss_h;
  float v[kRowsPerWarp][8];
#pragma unroll
  for (int j = 0; j < kRowsPerWarp; ++j) {
    if (l0 + j < a.L) {
      load8(src + static_cast<long>(l0 + j) * a.xs_l, v[j]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[j][i] = 0.f;
    }
  }
  // ring slot of token l: region_base + (off + l) mod region_len, with
  // l < L <= region_len and off < region_len, so one conditional subtract wraps
  auto slot_of = [&](int l) {
    const long ol = static_cast<long>(off) + l;
    return a.region_base + (ol >= a.region_len ? ol - a.region_len : ol);
  };
  if (MODE == kQuantI8Sym) {
    float amax[kRowsPerWarp];
#pragma unroll
    for (int j = 0; j < kRowsPerWarp; ++j) {
      float m = 0.f;  // fmaxf skips NaN, so every lane's value is a non-negative number
#pragma unroll
      for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[j][i]));
      // non-negative floats order like their bit patterns: one warp-wide integer max
      amax[j] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    }
    float mine = amax[0];
#pragma unroll
    for (int j = 1; j < kRowsPerWarp; ++j)
      if (lane == j) mine = amax[j];
    const float my_scale = __fdiv_rn(mine, 127.0f);
    const float my_rcp = __frcp_rn(my_scale);
#pragma unroll
    for (int j = 0; j < kRowsPerWarp; ++j) {
      const int l = l0 + j;
      if (l >= a.L) break;
      const float scale = __shfl_sync(0xffffffffu, my_scale, j);
      const float rcp = __shfl_sync(0xffffffffu, my_rcp, j);
      uint32_t packed[2] = {0u, 0u};
      if (amax[j] > 0.f) quant8_i8(v[j], scale, rcp, packed);
      const long slot = slot_of(l);
      *reinterpret_cast<uint2*>(qbase + slot * a.qs_c) = make_uint2(packed[0], packed[1]);
      if (lane == 0) static_cast<float*>(a.scale[which])[sbase + slot * a.ss_c] = scale;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kRowsPerWarp; ++j) {
      const int l = l0 + j;
      if (l >= a.L) break;
      // Reference scheme, each op rounded to the activation dtype:
      //   range = clamp(max - min, min=1e-5); scale = range / 255;
      //   zp = -min / scale; q = clamp(round(x / scale + zp), 0, 255)
      float mn = v[j][0], mx = v[j][0];
#pragma unroll
      for (int i = 1; i < 8; ++i) {
        mn = fminf(mn, v[j][i]);
        mx = fmaxf(mx, v[j][i]);
      }
      mn = warp_min(mn);
      mx = warp_max(mx);
      float range = to_act<Tin>(mx - mn);
      const float kMinRange = to_act<Tin>(1e-5f);
      if (range < 1e-5f) range = kMinRange;
      const float scale = to_act<Tin>(__fdiv_rn(range, 255.0f));
      const float zp = to_act<Tin>(__fdiv_rn(-mn, scale));
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float t1 = to_act<Tin>(__fdiv_rn(v[j][i], scale));
        const float t2 = to_act<Tin>(__fadd_rn(t1, zp));
        float r = rintf(t2);
        r = fminf(fmaxf(r, 0.f), 255.f);
        packed[i >> 2] |= (static_cast<uint32_t>(r) & 0xFFu) << (8 * (i & 3));
      }
      const long slot = slot_of(l);
      *reinterpret_cast<uint2*>(qbase + slot * a.qs_c) = make_uint2(packed[0], packed[1]);
      if (lane == 0) {
        const long sidx = sbase + slot * a.ss_c;
        store_act<Tin>(static_cast<Tin*>(a.scale[which]) + sidx, scale);
        store_act<Tin>(static_cast<Tin*>(a.zp[which]) + sidx, zp);
      }
    }
  }
}

// V pointers all null: quantize K alone (fused_quantize_store of one tensor)
bool kv_quant_k_only(const KvQuantDesc& d) { return !d.x[1] && !d.q[1] && !d.scale[1] && !d.zp[1]; }

}  // namespace

int validate_kv_quant(const KvQuantDesc& d) {
  if (d.D != kD) return set_error(RFX_E_INVAL, "kv_quant_append: head_dim must be 256");
  if (d.B <= 0 || d.H <= 0 || d.L < 0) return set_error(RFX_E_INVAL, "kv_quant_append: bad B/H/L");
  if (d.L == 0) return RFX_OK;  // nothing to append: the call is a no-op
  if (d.region_len <= 0 || d.region_base < 0 || d.region_off < 0 || d.L > d.region_len)
    return set_error(RFX_E_INVAL, "kv_quant_append: bad ring region");
  if (static_cast<long>(d.region_base) + d.region_len > d.capacity)
    return set_error(RFX_E_INVAL, "kv_quant_append: ring region exceeds capacity");
  if (d.mode != kQuantI8Sym && d.mode != kQuantU8Ref) return set_error(RFX_E_INVAL, "kv_quant_append: bad mode");
  if (d.in_dtype != kDtypeBF16 && d.in_dtype != kDtypeF32)
    return set_error(RFX_E_INVAL, "kv_quant_append: input dtype must be bf16 or f32");
  const int nw = kv_quant_k_only(d) ? 1 : 2;
  for (int w = 0; w < nw; ++w) {
    if (!d.x[w] || !d.q[w] || !d.scale[w] || (d.mode == kQuantU8Ref && !d.zp[w]))
      return set_error(RFX_E_INVAL, "kv_quant_append: null pointer");
    if ((reinterpret_cast<uintptr_t>(d.x[w]) & 15u) || (reinterpret_cast<uintptr_t>(d.q[w]) & 7u))
      return set_error(RFX_E_INVAL, "kv_quant_append: misaligned input/ring pointer");
  }
  const int esz = d.in_dtype == kDtypeBF16 ? 2 : 4;
  if (((d.xs_b | d.xs_h | d.xs_l) * esz) % 16 || (d.qs_b | d.qs_h | d.qs_c) % 8)
    return set_error(RFX_E_INVAL, "kv_quant_append: strides must keep 16-byte rows");
  if (static_cast<long>(d.B) * d.H > 65535)
    return set_error(RFX_E_INVAL, "kv_quant_append: B * H must be at most 65535");
  return RFX_OK;
}

int launch_kv_quant_append(const KvQuantDesc& d, cudaStream_t stream, bool pdl) {
  int rc = validate_kv_quant(d);
  if (rc || d.L == 0) return rc;
  const int nw = kv_quant_k_only(d) ? 1 : 2;

  QuantArgs a{};
  for (int w = 0; w < 2; ++w) {
    a.x[w] = d.x[w];
    a.q[w] = d.q[w];
    a.scale[w] = d.scale[w];
    a.zp[w] = d.zp[w];
  }
  a.xs_b = d.xs_b; a.xs_h = d.xs_h; a.xs_l = d.xs_l;
  a.qs_b = d.qs_b; a.qs_h = d.qs_h; a.qs_c = d.qs_c;
  a.ss_b = d.ss_b; a.ss_h = d.ss_h; a.ss_c = d.ss_c;
  a.B = d.B; a.H = d.H; a.L = d.L;
  a.region_base = d.region_base; a.region_off = d.region_off; a.region_len = d.region_len;

  constexpr int kRowsPerBlock = kWarpsPerBlock * kRowsPerWarp;
  dim3 grid(static_cast<unsigned>((d.L + kRowsPerBlock - 1) / kRowsPerBlock), static_cast<unsigned>(d.B * d.H), nw);
  dim3 block(kWarpsPerBlock * 32);
  void (*kern)(QuantArgs) = nullptr;
  if (d.in_dtype == kDtypeBF16)
    kern = d.mode == kQuantI8Sym ? kv_quant_append_kernel<__nv_bfloat16, kQuantI8Sym>
                                 : kv_quant_append_kernel<__nv_bfloat16, kQuantU8Ref>;
  else
    kern = d.mode == kQuantI8Sym ? kv_quant_append_kernel<float, kQuantI8Sym> : kv_quant_append_kernel<float, kQuantU8Ref>;
  return launch_kernel(reinterpret_cast<const void*>(kern), grid, block, 0, stream, pdl, 1, a);
}

}  // namespace rfx
