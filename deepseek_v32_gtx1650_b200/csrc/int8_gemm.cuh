// int8_gemm: block-scaled INT8 GEMM on the sm_100a tensor cores.
//
//   C[m, n] = sum_{kb < K/128} fp32( sum_{k in kb} A[m,k] * B[n,k] ) * (a_s[m,kb] * b_s[n/128, kb])
//
// Semantics: reference.py:18-24 (int8_gemm_ref, float64) and kernels.py:71-101 (fp32
// accumulation of the scaled per-block int32 partials). Operands are the reference layout:
// A [M, K] int8 and B [N, K] int8 ("nn.Linear" layout), both K-contiguous, which is exactly
// the K-major operand form tcgen05 reads; a_s [M, K/128], b_s [N/128, K/128] fp32.
//
// Design (one CTA per SM, persistent over 128 x BN output tiles):
//   warp 8      TMA producer: 128x128 A and BNx128 B tiles (SWIZZLE_128B) into a 4-stage ring.
//   warp 9      MMA issuer: per 128-K block, 4 x tcgen05.mma.kind::i8 (K = 32 each) into one of
//               two TMEM int32 accumulators (BN columns each), committed to the epilogue.
//   warps 0-7   promotion epilogue: for every K block, tcgen05.ld the int32 partial, convert,
//               multiply by a_s*b_s and accumulate in fp32 registers; refill the buffer with the
//               conversion bias so the MMA of K block kb+2 can reuse it. Warp w owns TMEM lanes
//               32*(w%4)..+31 (rows) and column half w/4.
// The int32 partials are pre-biased (common.cuh: kI32FloatBiasBits): the accumulator starts at
// bits(1.5*2^23), so after the MMA its bits read as the float 1.5*2^23 + partial, and a single
// exact FADD recovers fp32(partial). |partial| <= 128*127*127 < 2^21, well inside the exact range.
//
// Every mbarrier wait is bounded (common.cuh); on a timeout the CTA drains its in-flight TMA
// loads and MMAs, frees TMEM and returns, leaving an error word for dsv32_device_status().
#pragma once
#include "common.cuh"

namespace dsv32 {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBK = 128;
constexpr int kStages = 4;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (kEpiWarps + 4) * 32;  // + one warpgroup: producer, MMA, 2 idle
// Launch: 384 threads x 168 registers = 64512. setmaxnreg moves them to the epilogue:
// 2 warpgroups x 128 x 232 + 1 warpgroup x 128 x 40 = 64512 (and per sub-partition
// 232 + 232 + 40 = 504 <= 512).
constexpr uint32_t kEpiRegs = 232;
constexpr uint32_t kCtlRegs = 40;
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;

template <int BN>
struct Smem {
  static constexpr int kA = kBM * kBK;          // bytes per A stage
  static constexpr int kB = BN * kBK;           // bytes per B stage
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kA;
  static constexpr int kOffBar = kOffB + kStages * kB;
  // full[kStages], empty[kStages], tfull[2], tempty[2], mma_done
  static constexpr int kNumBars = 2 * kStages + 5;
  static constexpr int kOffTmem = kOffBar + 8 * kNumBars;
  static constexpr int kOffAbort = kOffTmem + 4;
  static constexpr int kBytes = kOffAbort + 4;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment (SWIZZLE_128B)
};

enum : uint32_t { kOutF32 = 0, kOutBF16 = 1, kOutF16 = 2 };

// Drain wait: bounded, ignores the abort flag (used only while winding down).
DSV32_DEV void drain_wait(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > DSV32_WAIT_LIMIT_CYCLES / 16) break;
  }
}

template <int BN, bool kPartials>
__global__ void __launch_bounds__(kThreads, 1)
    int8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const float* __restrict__ a_s, const float* __restrict__ b_s, void* __restrict__ C,
                     uint32_t out_kind, int M, int N, int K, int32_t* __restrict__ partials) {
  using L = Smem<BN>;
  constexpr int kCols = BN / 2;  // columns per epilogue thread
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);

  const uint32_t sA = base + L::kOffA;
  const uint32_t sB = base + L::kOffB;
  const uint32_t bar0 = base + L::kOffBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto tfull_bar = [&](int b) { return bar0 + 8u * (2 * kStages + b); };
  auto tempty_bar = [&](int b) { return bar0 + 8u * (2 * kStages + 2 + b); };
  const uint32_t mma_done_bar = bar0 + 8u * (2 * kStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffTmem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KG = K / kBK;
  const int num_m = (M + kBM - 1) / kBM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), kEpiWarps);
    }
    mbar_init(mma_done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tmem_alloc(smem_u32(tmem_slot), 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= kEpiWarps) {
    regs_dec<kCtlRegs>();
  }
  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int m0 = (t / num_n) * kBM;
        const int n0 = (t % num_n) * BN;
        for (int kb = 0; kb < KG; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, (KID_GEMM << 16) | 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), L::kA + L::kB);
          tma_load_2d(sA + stage * L::kA, &tmA, full_bar(stage), kb * kBK, m0);
          tma_load_2d(sB + stage * L::kB, &tmB, full_bar(stage), kb * kBK, n0);
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Wait for the last loads issued into each stage to land before the CTA can exit.
      for (int i = 0; i < kStages && i < issued; ++i) {
        if (--stage < 0) {
          stage = kStages - 1;
          phase ^= 1u;
        }
        drain_wait(full_bar(stage), phase);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_i8(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t u = 0;  // K blocks processed by this CTA (selects the TMEM buffer)
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        for (int kb = 0; kb < KG; ++kb, ++u) {
          const uint32_t buf = u & 1u;
          if (!mbar_wait(tempty_bar(buf), (u >> 1) & 1u, abort_flag, (KID_GEMM << 16) | 2) ||
              !mbar_wait(full_bar(stage), phase, abort_flag, (KID_GEMM << 16) | 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sA + stage * L::kA;
          const uint32_t b_addr = sB + stage * L::kB;
          const uint32_t d_tmem = tmem_base + buf * BN;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            umma_i8(d_tmem, make_sdesc(a_addr + 32 * k, 128), make_sdesc(b_addr + 32 * k, 128), idesc, 1u);
          }
          umma_commit(empty_bar(stage));
          umma_commit(tfull_bar(buf));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      umma_commit(mma_done_bar);
      drain_wait(mma_done_bar, 0);
    }
  } else if (warp < kEpiWarps) {
    regs_inc<kEpiRegs>();
    // ------------------------------------------------------------ promotion epilogue
    const int wq = warp & 3;   // TMEM lane quarter
    const int wh = warp >> 2;  // column half
    const uint32_t t_lane = tmem_base + (uint32_t(wq * 32) << 16) + uint32_t(wh * kCols);
    bool ok = true;
    // Arm both accumulators with the conversion bias.
#pragma unroll
    for (int b = 0; b < 2; ++b) {
#pragma unroll
      for (int c = 0; c < kCols / 32; ++c) tmem_fill32(t_lane + b * BN + c * 32, kI32FloatBiasBits);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(tempty_bar(0));
      mbar_arrive(tempty_bar(1));
    }
    uint32_t u = 0;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const int m0 = (t / num_n) * kBM;
      const int n0 = (t % num_n) * BN;
      const int row = m0 + wq * 32 + lane;
      const int col0 = n0 + wh * kCols;
      const bool row_ok = row < M;
      const bool cols_ok = col0 < N;  // N % 128 == 0: a half is either fully in or fully out
      const float* as_row = a_s + static_cast<int64_t>(row_ok ? row : 0) * KG;
      const float* bs_row = b_s + static_cast<int64_t>(cols_ok ? (col0 / 128) : 0) * KG;
      float2 acc[kCols / 2];
#pragma unroll
      for (int j = 0; j < kCols / 2; ++j) acc[j] = make_float2(0.f, 0.f);

      for (int kb = 0; kb < KG; ++kb, ++u) {
        const uint32_t buf = u & 1u;
        const float sa = row_ok ? __ldg(as_row + kb) : 0.f;
        const float sb = cols_ok ? __ldg(bs_row + kb) : 0.f;
        const float sc = sa * sb;
        const float2 sc2 = make_float2(sc, sc);
        const float2 nbias = make_float2(-kI32FloatBias, -kI32FloatBias);
        if (!mbar_wait_warp(tfull_bar(buf), (u >> 1) & 1u, abort_flag, (KID_GEMM << 16) | 4)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kCols / 32; ++c) {
          uint32_t r[32];
          const uint32_t ta = t_lane + buf * BN + c * 32;
          tmem_ld32(ta, r);
          tmem_fill32(ta, kI32FloatBiasBits);
          if constexpr (kPartials) {
            if (row_ok && cols_ok) {
              int32_t* p = partials + (static_cast<int64_t>(kb) * M + row) * N + col0 + c * 32;
#pragma unroll
              for (int j = 0; j < 32; ++j) p[j] = static_cast<int32_t>(r[j] - kI32FloatBiasBits);
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float2 v = make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
            v = __fadd2_rn(v, nbias);
            acc[c * 16 + j] = __ffma2_rn(v, sc2, acc[c * 16 + j]);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar(buf));
      }
      if (!ok) break;
      if (row_ok && cols_ok) {
        const int64_t off = static_cast<int64_t>(row) * N + col0;
        if (out_kind == kOutF32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(C) + off);
#pragma unroll
          for (int j = 0; j < kCols / 4; ++j)
            dst[j] = make_float4(acc[2 * j].x, acc[2 * j].y, acc[2 * j + 1].x, acc[2 * j + 1].y);
        } else if (out_kind == kOutBF16) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(C) + off);
#pragma unroll
          for (int j = 0; j < kCols / 8; ++j) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              __nv_bfloat162 h = __float22bfloat162_rn(acc[4 * j + i]);
              w[i] = *reinterpret_cast<uint32_t*>(&h);
            }
            dst[j] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(C) + off);
#pragma unroll
          for (int j = 0; j < kCols / 8; ++j) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              __half2 h = __float22half2_rn(acc[4 * j + i]);
              w[i] = *reinterpret_cast<uint32_t*>(&h);
            }
            dst[j] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    __syncwarp();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

}  // namespace gemm
}  // namespace dsv32
