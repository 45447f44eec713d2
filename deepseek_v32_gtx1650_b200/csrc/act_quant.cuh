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
//
// Per value the work stays on the FP32 pipe: amax with a NaN-propagating max, the exact quotient
// and its rounding by packed f32x2 multiplies, FMAs and adds whose result bits carry the int8
// (aq_quant_exact), and byte permutes to pack four results; no float -> int conversion and no
// division per value, no branch.
#pragma once
#include "common.cuh"

namespace dsv32 {

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

// max(a, b) that returns NaN when either input is NaN (torch.amax propagates NaN; fmaxf drops it).
DSV32_DEV float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
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

// fp32 bits of rint(fl(x / s)) + 1.5 * 2^23 through the IEEE division; NaN -> 0.
DSV32_DEV float aq_exact_bits(float x, float s) {
  const float v = rintf(__fdiv_rn(x, s));
  return (v == v) ? v + 12582912.0f : 12582912.0f;
}

// round_half_even(x / s) for EPL values of one group with scale s (|x| <= the group's amax), returned as
// the fp32 bits of q + 1.5 * 2^23 (low byte = q as int8), exactly and without a branch per value:
// with z = RN(1/s) (the correctly rounded reciprocal, once per group) and y = RN(x * z),
//   q = RN(y + RN(x - y * s) * z) = RN(x / s)
// (Markstein's theorem: y is within one ulp of x / s, so the remainder x - y * s is exact in one FMA,
// and one correction with a correctly rounded reciprocal gives the correctly rounded quotient; valid
// without overflow or underflow, which |q| <= 127.x and s >= 1e-4 / 127 rule out). RN(q + 1.5 * 2^23)
// then rounds q to an integer with ties to even; its low byte is the int8. Per pair of values one
// packed multiply, two packed FMAs and one packed add. A scale that is not finite (an infinity or
// NaN in the group) takes the IEEE division per value (aq_exact_bits: NaN -> 0).
template <int EPL>
DSV32_DEV void aq_quant_exact(const float (&f)[EPL], float sc, uint32_t (&q)[EPL]) {
  constexpr float kMagic = 12582912.0f;
  if (sc < INFINITY) {
    const float z = __frcp_rn(sc);
    const float2 z2 = make_float2(z, z), ns2 = make_float2(-sc, -sc), m2 = make_float2(kMagic, kMagic);
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
      const float2 x2 = make_float2(f[e], f[e + 1]);
      const float2 y = __fmul2_rn(x2, z2);
      const float2 r = __ffma2_rn(y, ns2, x2);   // x - y * s, exact
      const float2 qq = __ffma2_rn(r, z2, y);    // RN(x / s)
      const float2 big = __fadd2_rn(qq, m2);     // rint, ties to even, + 1.5 * 2^23
      q[e] = __float_as_uint(big.x);
      q[e + 1] = __float_as_uint(big.y);
    }
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) q[e] = __float_as_uint(aq_exact_bits(f[e], sc));
  }
}

// Low bytes of four quantised results (aq_quant_exact bits), in order, as one 32-bit word.
DSV32_DEV uint32_t aq_pack4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// EPL values of a group per lane (LPG = 128 / EPL lanes per group, 32 / LPG groups per warp slot),
// read as EPL * sizeof(T) / 16 consecutive 16-byte vectors; UNROLL group slots per iteration.
template <typename T, int EPL, int UNROLL>
__global__ void __launch_bounds__(256) act_quant_kernel(const T* __restrict__ x, int8_t* __restrict__ y,
                                                        float* __restrict__ s, int64_t num_groups,
                                                        int round_scale) {
  constexpr int LPG = 128 / EPL;
  constexpr int GPW = 32 / LPG;  // groups per warp-slot
  constexpr int NV = EPL * static_cast<int>(sizeof(T)) / 16;  // 16-byte vectors per lane
  constexpr int FPV = 16 / static_cast<int>(sizeof(T));        // values per vector
  static_assert(NV >= 1 && LPG >= 1 && LPG <= 32 && EPL % 4 == 0, "unsupported lane split");
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPG;     // which group of the slot this lane works on
  const int sl = lane % LPG;      // lane within the group
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t slots = (num_groups + GPW - 1) / GPW;
  pdl_wait();
  pdl_launch_dependents();

  for (int64_t base = warp * UNROLL; base < slots; base += nwarps * UNROLL) {
    // All loads of the lane are issued before any is used; the raw vectors stay packed in
    // registers until their group is processed.
    uint4 raw[UNROLL][NV];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t g = (base + u) * GPW + sub;
      const bool valid = (base + u) < slots && g < num_groups;
      const uint4* src = reinterpret_cast<const uint4*>(x + g * 128 + sl * EPL);
#pragma unroll
      for (int j = 0; j < NV; ++j) raw[u][j] = valid ? __ldcs(src + j) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t g = (base + u) * GPW + sub;
      const bool valid = (base + u) < slots && g < num_groups;
      float f[EPL];
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if constexpr (sizeof(T) == 4) {
          to_f32(make_float4(__uint_as_float(raw[u][j].x), __uint_as_float(raw[u][j].y),
                             __uint_as_float(raw[u][j].z), __uint_as_float(raw[u][j].w)),
                 *reinterpret_cast<float(*)[4]>(f + j * FPV));
        } else {
          to_f32(raw[u][j], *reinterpret_cast<float(*)[8]>(f + j * FPV), static_cast<T*>(nullptr));
        }
      }
      float a = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) a = max_nan(a, fabsf(f[e]));
#pragma unroll
      for (int o = LPG / 2; o > 0; o >>= 1) a = max_nan(a, __shfl_xor_sync(0xffffffffu, a, o));
      const float amax = max_nan(a, 1e-4f);  // NaN anywhere in the group -> NaN
      const float sc = aq_scale(amax, round_scale != 0);
      if (valid) {
        uint32_t qb[EPL];
        aq_quant_exact<EPL>(f, sc, qb);
        int8_t* dst = y + g * 128 + sl * EPL;
        if constexpr (EPL == 4) {
          __stcs(reinterpret_cast<unsigned int*>(dst), aq_pack4(qb[0], qb[1], qb[2], qb[3]));
        } else if constexpr (EPL == 8) {
          __stcs(reinterpret_cast<uint2*>(dst), make_uint2(aq_pack4(qb[0], qb[1], qb[2], qb[3]),
                                                           aq_pack4(qb[4], qb[5], qb[6], qb[7])));
        } else {
#pragma unroll
          for (int j = 0; j < EPL / 16; ++j)
            __stcs(reinterpret_cast<uint4*>(dst) + j,
                   make_uint4(aq_pack4(qb[16 * j + 0], qb[16 * j + 1], qb[16 * j + 2], qb[16 * j + 3]),
                              aq_pack4(qb[16 * j + 4], qb[16 * j + 5], qb[16 * j + 6], qb[16 * j + 7]),
                              aq_pack4(qb[16 * j + 8], qb[16 * j + 9], qb[16 * j + 10], qb[16 * j + 11]),
                              aq_pack4(qb[16 * j + 12], qb[16 * j + 13], qb[16 * j + 14], qb[16 * j + 15])));
        }
        if (sl == 0) s[g] = sc;
      }
    }
  }
}

}  // namespace dsv32

namespace dsv32 {

// ---------------------------------------------------------------- 16-bit input (bf16 / fp16)
// 16-bit input moves 60 % of fp32's bytes for the same work per value, so its kernel is leaner:
// one 128-value group per 16 lanes (8 values per lane, one 16-byte load), two groups per warp slot,
// UNROLL consecutive slots per warp iteration; the scale format is a template parameter; iterations
// whose slots are all complete run without validity tests, their loads and stores at constant
// offsets from one base pointer. (16-bit data is full of rounding ties: a value equal to amax / 2
// gives x / s = 63.5 up to the rounding of s, and about a third of the groups of normal bf16 data
// hold one, which is why the exact rounding has no near-tie test and fix-up branch.)

template <bool kRound>
DSV32_DEV float aq_scale_t(float amax) {
  return aq_scale(amax, kRound);
}

template <typename T, bool kRound>
DSV32_DEV void aq16_slot(const uint4& raw, uint2& out, float& sc) {
  float f[8];
  to_f32(raw, f, static_cast<T*>(nullptr));
  float a = max_nan(max_nan(max_nan(fabsf(f[0]), fabsf(f[1])), max_nan(fabsf(f[2]), fabsf(f[3]))),
                    max_nan(max_nan(fabsf(f[4]), fabsf(f[5])), max_nan(fabsf(f[6]), fabsf(f[7]))));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) a = max_nan(a, __shfl_xor_sync(0xffffffffu, a, o));
  sc = aq_scale_t<kRound>(max_nan(a, 1e-4f));  // NaN anywhere in the group -> NaN
  uint32_t q[8];
  aq_quant_exact<8>(f, sc, q);
  out = make_uint2(aq_pack4(q[0], q[1], q[2], q[3]), aq_pack4(q[4], q[5], q[6], q[7]));
}

template <typename T, bool kRound, int UNROLL>
__global__ void __launch_bounds__(256) act_quant16_kernel(const T* __restrict__ x, int8_t* __restrict__ y,
                                                          float* __restrict__ s, int64_t num_groups) {
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 4;  // group of the slot
  const int sl = lane & 15;   // lane within the group
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t full_slots = num_groups >> 1;  // slots holding two groups
  pdl_wait();
  pdl_launch_dependents();

  int64_t base = warp * UNROLL;
  for (; base + UNROLL <= full_slots; base += nwarps * UNROLL) {
    const int64_t g0 = base * 2 + sub;  // this lane's group in slot 0; slot u is 2u groups further
    const uint4* src = reinterpret_cast<const uint4*>(x + g0 * 128 + sl * 8);
    uint4 raw[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) raw[u] = __ldcs(src + u * 32);
    uint2 out[UNROLL];
    float sc[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) aq16_slot<T, kRound>(raw[u], out[u], sc[u]);
    uint2* dst = reinterpret_cast<uint2*>(y + g0 * 128 + sl * 8);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) __stcs(dst + u * 32, out[u]);
    if (sl == 0) {
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) s[g0 + 2 * u] = sc[u];
    }
  }
  // The warp's last, incomplete iteration (and an odd last group): one slot at a time, checked.
  const int64_t slots = (num_groups + 1) >> 1;
  for (int64_t sb = base; sb < base + UNROLL && sb < slots; ++sb) {
    const int64_t g = sb * 2 + sub;
    const bool valid = g < num_groups;
    const uint4 raw = valid ? __ldcs(reinterpret_cast<const uint4*>(x + g * 128 + sl * 8)) : make_uint4(0u, 0u, 0u, 0u);
    uint2 out;
    float sc;
    aq16_slot<T, kRound>(raw, out, sc);
    if (valid) {
      __stcs(reinterpret_cast<uint2*>(y + g * 128 + sl * 8), out);
      if (sl == 0) s[g] = sc;
    }
  }
}

}  // namespace dsv32
