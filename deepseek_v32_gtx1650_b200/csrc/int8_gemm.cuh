// int8_gemm: block-scaled INT8 GEMM on the sm_100a tensor cores.
//
//   C[m, n] = sum_{kb < K/128} fp32( sum_{k in kb} A[m,k] * B[n,k] ) * (a_s[m,kb] * b_s[n/128, kb])
//
// Semantics: reference.py:18-24 (int8_gemm_ref, float64) and kernels.py:71-101 (fp32
// accumulation of the scaled per-block int32 partials). Operands are the reference layout:
// A [M, K] int8 and B [N, K] int8 ("nn.Linear" layout), both K-contiguous, which is exactly
// the K-major operand form tcgen05 reads; a_s [M, K/128], b_s [N/128, K/128] fp32.
//
// Roles (one CTA per SM, 384 threads):
//   warp 8      TMA producer: 128x128 A and BNx128 B tiles (SWIZZLE_128B) into a 192 KB ring
//               (4 stages for BN = 256, 6 for BN = 128).
//   warp 9      MMA issuer: per 128-K block, 4 x tcgen05.mma.kind::i8 (K = 32 each) into one of
//               512 / BN TMEM int32 accumulators (BN columns each), committed to the epilogue.
//   warps 0-7   promotion epilogue: for every K block, tcgen05.ld the int32 partial, convert it
//               to fp32 (exact: |partial| <= 128*127*127 < 2^24), multiply by a_s*b_s and
//               accumulate in fp32 registers (packed f32x2 FMA), then release the TMEM buffer.
//               Warp w owns TMEM lanes 32*(w%4)..+31 (rows) and column half w/4. TMEM reads are
//               software-pipelined: the next 16-column chunk is in flight while the current one
//               is promoted. The first MMA of each K block overwrites the accumulator, so the
//               buffer needs no clearing between K blocks.
//
// Schedule (stream-K): the work is tiles x K-blocks "units", ordered tile-major. CTA c processes
// the contiguous unit range [U*c/G, U*(c+1)/G), so every SM gets the same number of K-blocks
// whatever the tile count. A range covers whole tiles (stored directly) and at most two partial
// tiles. A partial tile's fp32 accumulator goes to a workspace slot; the CTA that completes the
// tile last (atomic counter) adds the slots in ascending K order and stores C. No CTA ever waits
// for another. Without a workspace the kernel runs plain data-parallel tiles.
//
// Every mbarrier wait is bounded (common.cuh); on a timeout the CTA drains its in-flight TMA
// loads and MMAs, frees TMEM and returns, leaving an error word for dsv32_device_status().
#pragma once
#include "common.cuh"

namespace dsv32 {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBK = 128;
// Epilogue warps per CTA (EW = 8 or 16), the kernel's template parameter. The CTA is EW epilogue
// warps plus one warpgroup (producer, MMA issuer, 2 idle).
constexpr int kEpiWarps = 8;        // default
constexpr int kMaxEpiWarps = 16;    // counters per tile in the workspace (either layout fits)
__host__ __device__ constexpr int threads_for(int ew) { return (ew + 4) * 32; }
constexpr int kThreads = threads_for(kEpiWarps);
// setmaxnreg moves registers from the control warpgroup to the epilogue. It draws on the registers
// the CTA was launched with (threads x registers per thread at launch, 65536 / threads rounded down
// to 8), not on the SM's file: the split must fit that total or the increasing warps wait forever.
//   EW = 8:  384 threads x 168 = 64512 >= 2 x 128 x 216 + 128 x 72   (per sub-partition 504 <= 512)
//   EW = 16: 640 threads x  96 = 61440 >= 4 x 128 x 112 + 128 x 32   (per sub-partition 480 <= 512)
__host__ __device__ constexpr uint32_t epi_regs(int ew) { return ew == 8 ? 216u : 112u; }
__host__ __device__ constexpr uint32_t ctl_regs(int ew) { return ew == 8 ? 72u : 32u; }
__host__ __device__ constexpr int launch_regs(int ew) { return (65536 / threads_for(ew)) & ~7; }
static_assert(epi_regs(8) * 8 * 32 + ctl_regs(8) * 4 * 32 <= threads_for(8) * launch_regs(8),
              "register split exceeds the launch allocation");
static_assert(epi_regs(16) * 16 * 32 + ctl_regs(16) * 4 * 32 <= threads_for(16) * launch_regs(16),
              "register split exceeds the launch allocation");
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;

template <int BN>
struct Smem {
  static constexpr int kStages = (BN == 256) ? 4 : 6;  // operand ring depth (192 KB either way)
  static constexpr int kTB = 512 / BN;                 // TMEM accumulator buffers (all 512 columns)
  static constexpr int kA = kBM * kBK;          // bytes per A stage
  static constexpr int kB = BN * kBK;           // bytes per B stage
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kA;
  static constexpr int kOffBar = kOffB + kStages * kB;
  // full[kStages], empty[kStages], tfull[kTB], tempty[kTB], mma_done
  static constexpr int kNumBars = 2 * kStages + 2 * kTB + 1;
  static constexpr int kOffTmem = kOffBar + 8 * kNumBars;
  static constexpr int kOffAbort = kOffTmem + 4;
  static constexpr int kBytes = kOffAbort + 4;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment (SWIZZLE_128B)
};

enum : uint32_t { kOutF32 = 0, kOutBF16 = 1, kOutF16 = 2 };

// Workspace layout (bytes): [counters: tiles_cap x 16 int32 (one per tile and epilogue warp); a fixed capacity per
// workspace, so the counters never share bytes with slot data whatever the problem shape]
// [2 * grid slots of slot_rows x BN fp32, column-major]. Slot 2c holds CTA c's first segment, slot
// 2c+1 its last one; slot_rows = min(128, M rounded up to 32) (rows past M are never written).
// The counters must be zero before the first launch; every completed launch leaves them zero.
constexpr int64_t kMaxSplitTiles = 65536;  // counter capacity of caller-provided workspaces
__host__ __device__ constexpr int64_t counter_bytes(int64_t tiles_cap) { return tiles_cap * kMaxEpiWarps * 4; }
__host__ __device__ inline int slot_rows_for(int64_t m) {
  return static_cast<int>(m >= kBM ? kBM : ((m + 31) / 32) * 32);
}
__host__ __device__ inline int64_t workspace_bytes(int BN, int grid, int64_t tiles_cap, int slot_rows) {
  return counter_bytes(tiles_cap) + int64_t(2) * grid * slot_rows * BN * 4;
}

struct Sched {
  int num_n, KG, num_tiles, grid;
  long long U;  // total units = num_tiles * KG
  bool split;   // stream-K (needs a workspace) or data-parallel tiles

  DSV32_DEV long long ubeg(int c) const { return (U * c) / grid; }
  DSV32_DEV int cta_of(long long u) const {
    int c = static_cast<int>((u * grid) / U);
    while (c + 1 < grid && ubeg(c + 1) <= u) ++c;
    while (c > 0 && ubeg(c) > u) --c;
    return c;
  }
};

// Iterates this CTA's segments: (tile, kb0, kb1, first-segment flag).
struct SegIter {
  const Sched& s;
  long long u, u1;  // stream-K range
  int t;            // data-parallel tile cursor
  bool first;
  DSV32_DEV explicit SegIter(const Sched& sc) : s(sc), first(true) {
    if (s.split) {
      u = s.ubeg(blockIdx.x);
      u1 = s.ubeg(blockIdx.x + 1);
    } else {
      t = blockIdx.x;
    }
  }
  DSV32_DEV bool next(int& tile, int& kb0, int& kb1, bool& is_first) {
    is_first = first;
    first = false;
    if (s.split) {
      if (u >= u1) return false;
      tile = static_cast<int>(u / s.KG);
      kb0 = static_cast<int>(u % s.KG);
      kb1 = static_cast<int>(min(static_cast<long long>(s.KG), kb0 + (u1 - u)));
      u += kb1 - kb0;
      return true;
    }
    if (t >= s.num_tiles) return false;
    tile = t;
    kb0 = 0;
    kb1 = s.KG;
    t += gridDim.x;
    return true;
  }
};

// Drain wait: bounded, ignores the abort flag (used only while winding down).
DSV32_DEV void drain_wait(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > DSV32_WAIT_LIMIT_CYCLES / 16) break;
  }
}

// acc[0..W/2) += float(partial) * sc for W columns (float2 pairs); the int32 -> fp32 conversion
// is exact for these magnitudes.
template <int W>
DSV32_DEV void promote(const uint32_t (&r)[W], float2* acc, float2 sc2) {
#pragma unroll
  for (int j = 0; j < W / 2; ++j) {
    const float2 v = make_float2(static_cast<float>(static_cast<int32_t>(r[2 * j])),
                                 static_cast<float>(static_cast<int32_t>(r[2 * j + 1])));
    acc[j] = __ffma2_rn(v, sc2, acc[j]);
  }
}

template <int kCols>
DSV32_DEV void store_row(const float2 (&acc)[kCols / 2], void* C, uint32_t out_kind, int64_t off) {
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

template <int BN, bool kPartials, int EW = kEpiWarps>
__global__ void __launch_bounds__(threads_for(EW), 1)
    int8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const float* __restrict__ a_s, const float* __restrict__ b_s, void* __restrict__ C,
                     uint32_t out_kind, int M, int N, int K, int32_t* __restrict__ partials,
                     uint8_t* __restrict__ workspace, int ws_tiles_cap, int slot_rows) {
  static_assert(EW == 8 || EW == 16, "8 or 16 epilogue warps");
  using L = Smem<BN>;
  constexpr int kCols = BN / (EW / 4);  // columns per epilogue thread (EW / 4 column parts)
  constexpr int kProducer = EW, kMma = EW + 1;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);

  const uint32_t sA = base + L::kOffA;
  const uint32_t sB = base + L::kOffB;
  const uint32_t bar0 = base + L::kOffBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  constexpr int kStages = L::kStages;
  constexpr int kTB = L::kTB;
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto tfull_bar = [&](int b) { return bar0 + 8u * (2 * kStages + b); };
  auto tempty_bar = [&](int b) { return bar0 + 8u * (2 * kStages + kTB + b); };
  const uint32_t mma_done_bar = bar0 + 8u * (2 * kStages + 2 * kTB);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffTmem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  Sched sch;
  sch.KG = K / kBK;
  sch.num_n = (N + BN - 1) / BN;
  sch.num_tiles = ((M + kBM - 1) / kBM) * sch.num_n;
  sch.grid = gridDim.x;
  sch.U = static_cast<long long>(sch.num_tiles) * sch.KG;
  sch.split = workspace != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < kTB; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), EW);
    }
    mbar_init(mma_done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMma) tmem_alloc(smem_u32(tmem_slot), kTB * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // no global memory access before this point
  pdl_launch_dependents();

  if (warp >= EW) {
    regs_dec<ctl_regs(EW)>();
  }
  if (warp == kProducer) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      SegIter it(sch);
      int tile, kb0, kb1;
      bool first;
      while (ok && it.next(tile, kb0, kb1, first)) {
        const int m0 = (tile / sch.num_n) * kBM;
        const int n0 = (tile % sch.num_n) * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
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
  } else if (warp == kMma) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_i8(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t u = 0;  // K blocks processed by this CTA (selects the TMEM buffer)
      bool ok = true;
      SegIter it(sch);
      int tile, kb0, kb1;
      bool first;
      while (ok && it.next(tile, kb0, kb1, first)) {
        for (int kb = kb0; kb < kb1; ++kb, ++u) {
          const uint32_t buf = u % kTB;
          if (!mbar_wait(tempty_bar(buf), (u / kTB) & 1u, abort_flag, (KID_GEMM << 16) | 2) ||
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
            umma_i8(d_tmem, make_sdesc(a_addr + 32 * k, 128), make_sdesc(b_addr + 32 * k, 128), idesc,
                    k > 0 ? 1u : 0u);  // the K block's first MMA overwrites
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
  } else if (warp < EW) {
    regs_inc<epi_regs(EW)>();
    // ------------------------------------------------------------ promotion epilogue
    const int wq = warp & 3;   // TMEM lane quarter
    const int wh = warp >> 2;  // column part (of EW / 4)
    const int r_local = wq * 32 + lane;  // row within the tile
    const uint32_t t_lane = tmem_base + (uint32_t(wq * 32) << 16) + uint32_t(wh * kCols);
    int* counters = reinterpret_cast<int*>(workspace);
    float* slots = workspace ? reinterpret_cast<float*>(workspace + counter_bytes(ws_tiles_cap)) : nullptr;
    const int64_t slot_floats = static_cast<int64_t>(slot_rows) * BN;
    bool ok = true;
    // Both accumulators start free.
    __syncwarp();
    if (lane == 0) {
      for (int b = 0; b < kTB; ++b) mbar_arrive(tempty_bar(b));
    }
    uint32_t u = 0;
    SegIter it(sch);
    int tile, kb0, kb1;
    bool first_seg;
    while (ok && it.next(tile, kb0, kb1, first_seg)) {
      const int m0 = (tile / sch.num_n) * kBM;
      const int n0 = (tile % sch.num_n) * BN;
      const int row = m0 + r_local;
      const int col0 = n0 + wh * kCols;
      const bool row_ok = row < M;
      const bool cols_ok = col0 < N;  // N % 128 == 0: a half is either fully in or fully out
      const float* as_row = a_s + static_cast<int64_t>(row_ok ? row : 0) * sch.KG;
      const float* bs_row = b_s + static_cast<int64_t>(cols_ok ? (col0 / 128) : 0) * sch.KG;
      float2 acc[kCols / 2];
#pragma unroll
      for (int j = 0; j < kCols / 2; ++j) acc[j] = make_float2(0.f, 0.f);

      float sa_next = row_ok ? __ldg(as_row + kb0) : 0.f;
      float sb_next = cols_ok ? __ldg(bs_row + kb0) : 0.f;
      for (int kb = kb0; kb < kb1; ++kb, ++u) {
        const uint32_t buf = u % kTB;
        const float sc = sa_next * sb_next;
        if (kb + 1 < kb1) {  // prefetch the next block's scales
          sa_next = row_ok ? __ldg(as_row + kb + 1) : 0.f;
          sb_next = cols_ok ? __ldg(bs_row + kb + 1) : 0.f;
        }
        const float2 sc2 = make_float2(sc, sc);
        if (!mbar_wait_warp(tfull_bar(buf), (u / kTB) & 1u, abort_flag, (KID_GEMM << 16) | 4)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = t_lane + buf * BN;
        // TMEM reads are software-pipelined one chunk ahead; 32-column chunks when the 64
        // accumulators of a BN=128 tile leave room for two of them, else 16 columns (always 16 with
        // 16 epilogue warps, whose threads have 112 registers).
        constexpr int kCW = (EW == 8 && kCols <= 64) ? 32 : 16;
        uint32_t ra[kCW], rb[kCW];
        tmem_ld_async<kCW>(tb, ra);
        tmem_wait_ld<kCW>(ra);
#pragma unroll
        for (int c = 0; c < kCols / kCW; ++c) {
          uint32_t(&cur)[kCW] = (c & 1) ? rb : ra;
          uint32_t(&nxt)[kCW] = (c & 1) ? ra : rb;
          if (c + 1 < kCols / kCW) tmem_ld_async<kCW>(tb + (c + 1) * kCW, nxt);  // in flight during promote
          if constexpr (kPartials) {
            if (row_ok && cols_ok) {
              int32_t* p = partials + (static_cast<int64_t>(kb) * M + row) * N + col0 + c * kCW;
#pragma unroll
              for (int j = 0; j < kCW; ++j) p[j] = static_cast<int32_t>(cur[j]);
            }
          }
          promote<kCW>(cur, acc + c * (kCW / 2), sc2);
          if (c + 1 < kCols / kCW) tmem_wait_ld<kCW>(nxt);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar(buf));
      }
      if (!ok) break;

      const bool full_tile = (kb0 == 0 && kb1 == sch.KG);
      const int64_t off = static_cast<int64_t>(row) * N + col0;
      if (full_tile) {
        if (row_ok && cols_ok) store_row<kCols>(acc, C, out_kind, off);
        continue;
      }
      // Partial tile: publish this warp's 32 rows x kCols of the segment; the warp that completes
      // this sub-tile last (one counter per tile and warp) reduces and stores. Warp-local: no
      // barrier across warps, so an aborting warp can never strand the others.
      const int slot = 2 * blockIdx.x + (first_seg ? 0 : 1);
      float* my_slot = slots + slot * slot_floats + static_cast<int64_t>(wh) * kCols * slot_rows;
      if (row_ok && cols_ok) {
#pragma unroll
        for (int j = 0; j < kCols / 2; ++j) {  // column-major slot: lanes write consecutive rows
          __stcg(my_slot + (2 * j) * slot_rows + r_local, acc[j].x);
          __stcg(my_slot + (2 * j + 1) * slot_rows + r_local, acc[j].y);
        }
      }
      __threadfence();
      __syncwarp();
      const long long t_u0 = static_cast<long long>(tile) * sch.KG;
      const int c_first = sch.cta_of(t_u0);
      const int c_last = sch.cta_of(t_u0 + sch.KG - 1);
      int is_last = 0;
      if (lane == 0) {
        int* ctr = counters + static_cast<int64_t>(tile) * kMaxEpiWarps + warp;
        const int prev = atomicAdd(ctr, 1);
        is_last = (prev == c_last - c_first);
        if (is_last) *ctr = 0;  // ready for the next launch
      }
      is_last = __shfl_sync(0xffffffffu, is_last, 0);
      if (!is_last) continue;
      __threadfence();
      if (!(row_ok && cols_ok)) continue;
      // Every contributor (this one included) has written its slot: sum them in ascending K order
      // so the result does not depend on which CTA arrived last.
#pragma unroll
      for (int j = 0; j < kCols / 2; ++j) acc[j] = make_float2(0.f, 0.f);
      for (int cc = c_first; cc <= c_last; ++cc) {
        const int first_tile_of_cc = static_cast<int>(sch.ubeg(cc) / sch.KG);
        const int s = 2 * cc + (first_tile_of_cc == tile ? 0 : 1);
        const float* ps = slots + s * slot_floats + static_cast<int64_t>(wh) * kCols * slot_rows;
#pragma unroll
        for (int j = 0; j < kCols / 2; ++j) {
          const float2 v = make_float2(__ldcg(ps + (2 * j) * slot_rows + r_local),
                                       __ldcg(ps + (2 * j + 1) * slot_rows + r_local));
          acc[j] = __fadd2_rn(acc[j], v);
        }
      }
      store_row<kCols>(acc, C, out_kind, off);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMma) {
    __syncwarp();
    tmem_dealloc(tmem_base, kTB * BN);
  }
}

}  // namespace gemm
}  // namespace dsv32
