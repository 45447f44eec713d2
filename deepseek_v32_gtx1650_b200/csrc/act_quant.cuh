// act_quant: per 128-value group, amax -> fp32 scale (or ue8m0 power of two) -> int8.
//
// Semantics follow reference.py:8-15 (act_quant_ref) and kernels.py:37-52 exactly:
//   amax = max(max|x|, 1e-4)                 (fp32; the floor is fl32(1e-4))
//   s    = amax * fl32(1/127)                 (an fp32 multiply, not a division)
//   ue8m0: s = 2^ceil(log2 s), with log2 rounded to fp32 as torch's CPU log2 does
//   y    = clamp(round_half_even(x / s), -127, 127)   (IEEE fp32 division)
//
// Layout: x [rows, N] contiguous with N % 128 == 0 is a flat sequence of G = rows*N/128
// groups; group g covers x[128g : 128g+128], y[128g : 128g+128] and s[g]. So the kernel is a
// 1-D grid-stride loop over groups, independent of rows/N.
//
// Mapping: one group = 256 or 512 contiguous bytes, read as 16-byte vectors by
// 16 (bf16/fp16) or 32 (fp32) lanes; amax by xor-shuffles inside that lane group. Each
// warp handles UNROLL consecutive group-slots per iteration so several 16-byte loads
// are in flight per lane (HBM latency hiding).
#pragma once
#include "common.cuh"

namespace dsv32 {

template <typename T>
struct AqTraits;
template <>
struct AqTraits<float> {
  static constexpr int kLanesPerGroup = 32;  // 32 lanes x 4 fp32
  static constexpr int kElemsPerLane = 4;
};
template <>
struct AqTraits<__nv_bfloat16> {
  static constexpr int kLanesPerGroup = 16;  // 16 lanes x 8 bf16
  static constexpr int kElemsPerLane = 8;
};
template <>
struct AqTraits<__half> {
  static constexpr int kLanesPerGroup = 16;
  static constexpr int kElemsPerLane = 8;
};

DSV32_DEV void to_f32(const float4& v, float (&f)[4]) {
  f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
}
DSV32_DEV void to_f32(const uint4& v, float (&f)[8], __nv_bfloat16*) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
DSV32_DEV void to_f32(const uint4& v, float (&f)[8], __half*) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 p = __half22float2(h);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

// fp32 scale from the group amax (already floored), both formats.
DSV32_DEV float aq_scale(float amax, bool round_scale) {
  float s = amax * (1.0f / 127.0f);  // fl32(1/127) times fl32(amax), one fp32 rounding
  if (round_scale) {
    if (isfinite(s)) {
      // torch's CPU fp32 log2 returns the correctly rounded fp32 of log2(s): compute it in
      // double and round once. Then 2^ceil(.) is an exact power of two (|exp| < 127 here).
      const float l = static_cast<float>(log2(static_cast<double>(s)));
      const int e = static_cast<int>(ceilf(l));
      s = __int_as_float((e + 127) << 23);
    }
  }
  return s;
}

// round_half_even(x / s) for |x| <= amax, s = amax-derived scale (|x / s| <= 127 + tiny).
// Exact fast path: q = x * rcp_rn(s) is within 2^-15 of fl(x / s) for |q| < 128 (two correctly rounded
// steps, 2^-23 relative), so rint(q) == rint(fl(x / s)) unless q lies within 2^-14 of a half
// integer; those (about 1 in 8000) take the IEEE division. NaN converts to 0.
DSV32_DEV int aq_quant1(float x, float s, float r) {
  const float q = x * r;
  const float n = rintf(q);
  float v = n;
  if (fabsf(q - n) > 0.5f - 6.103515625e-05f) v = rintf(__fdiv_rn(x, s));  // near a tie
  return __float2int_rn(v);  // |v| <= 127: no clamp needed
}

template <typename T, int UNROLL>
__global__ void __launch_bounds__(256) act_quant_kernel(const T* __restrict__ x, int8_t* __restrict__ y,
                                                        float* __restrict__ s, int64_t num_groups,
                                                        int round_scale) {
  using Tr = AqTraits<T>;
  constexpr int LPG = Tr::kLanesPerGroup;
  constexpr int EPL = Tr::kElemsPerLane;
  constexpr int GPW = 32 / LPG;  // groups per warp-slot
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPG;     // which group of the slot this lane works on
  const int sl = lane % LPG;      // lane within the group
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t slots = (num_groups + GPW - 1) / GPW;

  for (int64_t base = warp * UNROLL; base < slots; base += nwarps * UNROLL) {
    float f[UNROLL][EPL];
    bool valid[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t g = (base + u) * GPW + sub;
      valid[u] = (base + u) < slots && g < num_groups;
      if (valid[u]) {
        if constexpr (sizeof(T) == 4) {
          const float4 v = __ldcs(reinterpret_cast<const float4*>(x + g * 128) + sl);
          to_f32(v, reinterpret_cast<float(&)[4]>(f[u]));
        } else {
          const uint4 v = __ldcs(reinterpret_cast<const uint4*>(x + g * 128) + sl);
          to_f32(v, reinterpret_cast<float(&)[8]>(f[u]), static_cast<T*>(nullptr));
        }
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) f[u][e] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      float a = 0.f;
      bool nan = false;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        a = fmaxf(a, fabsf(f[u][e]));
        nan |= isnan(f[u][e]);
      }
#pragma unroll
      for (int o = LPG / 2; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
      // torch's amax propagates NaN while fmaxf drops it: detect NaN per group explicitly.
      const unsigned nan_lanes = __ballot_sync(0xffffffffu, nan);
      const unsigned group_lanes = (LPG == 32) ? 0xffffffffu : (0xFFFFu << (sub * 16));
      float amax = fmaxf(a, 1e-4f);
      if (nan_lanes & group_lanes) amax = __int_as_float(0x7fc00000);
      const float sc = aq_scale(amax, round_scale != 0);
      const float rc = __frcp_rn(sc);
      if (valid[u]) {
        const int64_t g = (base + u) * GPW + sub;
        if constexpr (EPL == 4) {
          char4 q;
          q.x = static_cast<int8_t>(aq_quant1(f[u][0], sc, rc));
          q.y = static_cast<int8_t>(aq_quant1(f[u][1], sc, rc));
          q.z = static_cast<int8_t>(aq_quant1(f[u][2], sc, rc));
          q.w = static_cast<int8_t>(aq_quant1(f[u][3], sc, rc));
          __stcs(reinterpret_cast<char4*>(y + g * 128) + sl, q);
        } else {
          uint32_t w0 = 0, w1 = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) w0 |= (uint32_t(uint8_t(aq_quant1(f[u][e], sc, rc))) << (8 * e));
#pragma unroll
          for (int e = 0; e < 4; ++e) w1 |= (uint32_t(uint8_t(aq_quant1(f[u][4 + e], sc, rc))) << (8 * e));
          __stcs(reinterpret_cast<uint2*>(y + g * 128) + sl, make_uint2(w0, w1));
        }
        if (sl == 0) s[g] = sc;
      }
    }
  }
}

}  // namespace dsv32
