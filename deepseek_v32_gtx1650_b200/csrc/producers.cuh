// Producers of the hot path's int8 operands (the steps either side of the kernels):
//
// rotate_quant: the lightning indexer's q / k producer (hadamard_quant.py:63-103). Each 128-value
//   vector is rotated by the 128-point Walsh-Hadamard transform scaled by 128^-1/2, then quantised
//   with one scale per vector: s = max(amax, 1e-4) * fl32(1/127), y = clamp(rint(x / s), -127, 127).
//   The rotation is the butterfly form of hadamard_quant.py:54-81 (stages of stride 1, 2, ..., 64,
//   each (a, b) -> (a + b, a - b), then one multiply by fl32(128^-1/2)), in fp32 like the
//   reference's fused kernels; hadamard_quant.py:106-110 (float64) is the oracle, and the
//   reference's own bar applies (test_hadamard.py:20-27: int8 values equal except off-by-one where
//   fp32 and fp64 round a tie apart, scales within 1e-5).
//   Layout: 8 lanes per vector, 16 consecutive values per lane: stages of stride 1-8 stay in the
//   lane's registers, strides 16, 32, 64 are lane shuffles (xor 1, 2, 4).
//   With s_mul, s[r] = s_mul[r] * scale instead (the indexer folds its query scales into the head
//   weights, bench_indexer_e2e.py:55, without a separate elementwise kernel).
//
// weight_quant: the GEMM's B operand (test_kernels.py:80-82, bench.py:43-44): per 128 x 128 block
//   of W [N, K], s = max(amax, 1e-4) / 127 (an fp32 division), y = clamp(rint(x / s), -127, 127);
//   scales [N/128, K/128]. One CTA of 512 threads per block; each thread keeps 32 values in registers.
//
// Both use act_quant's branch-free exact rounding (aq_quant_exact): rint(fl(x / s)) from the
// correctly rounded reciprocal and one exact-remainder correction per value, valid for any normal
// scale s with |x / s| <= 127 + tiny.
#pragma once
#include "act_quant.cuh"

namespace dsv32 {

constexpr int kRqThreads = 256;
constexpr int kWqThreads = 512;

// 16 consecutive values of a 128-vector (16-bit or fp32 source) into fp32 registers.
template <typename T>
DSV32_DEV void load16(const T* src, float (&v)[16]) {
  if constexpr (sizeof(T) == 4) {
    const float4* p = reinterpret_cast<const float4*>(src);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 f = __ldcs(p + j);
      v[4 * j] = f.x;
      v[4 * j + 1] = f.y;
      v[4 * j + 2] = f.z;
      v[4 * j + 3] = f.w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int j = 0; j < 2; ++j) to_f32(__ldcs(p + j), *reinterpret_cast<float(*)[8]>(v + 8 * j), static_cast<T*>(nullptr));
  }
}

// Low bytes of 16 quantised values as one 16-byte vector.
DSV32_DEV uint4 pack16(const uint32_t (&q)[16]) {
  return make_uint4(aq_pack4(q[0], q[1], q[2], q[3]), aq_pack4(q[4], q[5], q[6], q[7]),
                    aq_pack4(q[8], q[9], q[10], q[11]), aq_pack4(q[12], q[13], q[14], q[15]));
}

template <typename T>
__global__ void __launch_bounds__(kRqThreads, 4) rotate_quant_kernel(const T* __restrict__ x, int8_t* __restrict__ y,
                                                                   float* __restrict__ s, int64_t rows, int rotate,
                                                                   const float* __restrict__ s_mul) {
  constexpr int LPV = 8;          // lanes per vector
  constexpr int VPW = 32 / LPV;   // vectors per warp slot
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPV;
  const int sl = lane % LPV;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t base = warp * VPW; base < rows; base += nwarps * VPW) {
    const int64_t row = base + sub;
    const bool valid = row < rows;
    float v[16];
    if (valid) {
      load16(x + row * 128 + sl * 16, v);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.f;
    }
    if (rotate) {
      // strides 1, 2, 4, 8: pairs inside this lane's 16 values, two butterflies per packed f32x2
      // add (a + b) and packed fma (b * -1 + a = a - b, one rounding like the subtraction)
      const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
      for (int st = 1; st < 16; st <<= 1) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if ((i & st) == 0 && ((i / st) & 2) == 0) {  // butterflies (i, i + st) and (j, j + st), j = i + 2 st
            const int j = (st == 8) ? i + 1 : i + 2 * st;
            if (st == 8 && (i & 1)) continue;
            const float2 a = make_float2(v[i], v[j]), b = make_float2(v[i + st], v[j + st]);
            const float2 sum = __fadd2_rn(a, b), dif = __ffma2_rn(b, neg1, a);
            v[i] = sum.x;
            v[j] = sum.y;
            v[i + st] = dif.x;
            v[j + st] = dif.y;
          }
        }
      }
      // strides 16, 32, 64: the partner value sits in lane sl ^ m of the same vector; the low lane
      // keeps v + o and the high lane o - v, both as fma(sign, v, o) (exact sign, one rounding)
#pragma unroll
      for (int m = 1; m < LPV; m <<= 1) {
        const float sg = (sl & m) ? -1.f : 1.f;
        const float2 sg2 = make_float2(sg, sg);
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float2 o = make_float2(__shfl_xor_sync(0xffffffffu, v[i], m), __shfl_xor_sync(0xffffffffu, v[i + 1], m));
          const float2 r = __ffma2_rn(make_float2(v[i], v[i + 1]), sg2, o);
          v[i] = r.x;
          v[i + 1] = r.y;
        }
      }
      constexpr float kInvSqrt128 = 0.08838834764831845f;  // fl32(128^-1/2)
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] *= kInvSqrt128;
    }
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) a = max_nan(a, fabsf(v[i]));
#pragma unroll
    for (int o = LPV / 2; o > 0; o >>= 1) a = max_nan(a, __shfl_xor_sync(0xffffffffu, a, o));
    const float sc = max_nan(a, 1e-4f) * (1.0f / 127.0f);
    if (valid) {
      uint32_t q[16];
      aq_quant_exact<16>(v, sc, q);
      __stcs(reinterpret_cast<uint4*>(y + row * 128 + sl * 16), pack16(q));
      // s_mul: the indexer's head weights, which take the per-vector query scale (w * qs,
      // bench_indexer_e2e.py:55: one fp32 rounding, as the reference's product)
      if (sl == 0) s[row] = s_mul ? __ldg(s_mul + row) * sc : sc;
    }
  }
}

// One CTA per 128 x 128 block of W [n, k]: thread t holds row t / 4, the 16-value chunks t % 4 and
// t % 4 + 4 of it (four threads read a row's 128 values as two contiguous 256-byte runs).
template <typename T>
__global__ void __launch_bounds__(kWqThreads, 2) weight_quant_kernel(const T* __restrict__ w, int8_t* __restrict__ wq,
                                                                  float* __restrict__ ws, int64_t n, int64_t k) {
  __shared__ float red[kWqThreads / 32];
  const int tid = threadIdx.x;
  const int64_t kb_count = k / 128;
  const int64_t nb = blockIdx.x / kb_count;
  const int64_t kb = blockIdx.x % kb_count;
  const int64_t row = nb * 128 + tid / 4;
  const int64_t col = kb * 128 + (tid % 4) * 16;
  pdl_wait();
  pdl_launch_dependents();
  float v[32];
#pragma unroll
  for (int j = 0; j < 2; ++j) load16(w + row * k + col + 64 * j, *reinterpret_cast<float(*)[16]>(v + 16 * j));
  float a = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) a = max_nan(a, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = max_nan(a, __shfl_xor_sync(0xffffffffu, a, o));
  if ((tid & 31) == 0) red[tid >> 5] = a;
  __syncthreads();
  a = red[0];
#pragma unroll
  for (int i = 1; i < kWqThreads / 32; ++i) a = max_nan(a, red[i]);
  const float sc = __fdiv_rn(max_nan(a, 1e-4f), 127.0f);
  uint32_t q[16];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    aq_quant_exact<16>(*reinterpret_cast<const float(*)[16]>(v + 16 * j), sc, q);
    *reinterpret_cast<uint4*>(wq + row * k + col + 64 * j) = pack16(q);
  }
  if (tid == 0) ws[nb * kb_count + kb] = sc;
}

}  // namespace dsv32
