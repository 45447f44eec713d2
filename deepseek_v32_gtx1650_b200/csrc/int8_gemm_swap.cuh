// int8_gemm for decode-sized m (m <= 64): the same block-scaled GEMM as int8_gemm.cuh with the
// operands swapped on the tensor cores.
//
//   C^T[n, m] = sum_kb fp32( B_kb[n, :] . A_kb[m, :] ) * (b_s[n/128, kb] * a_s[m, kb])
//
// Semantics are those of int8_gemm.cuh (reference.py:18-24, kernels.py:71-101); only the mapping
// differs. With 128-row A tiles a handful of tokens would fill a quarter (or less) of every MMA and
// every TMEM read with padding, and the promotion epilogue would walk eight dependent 16-column TMEM
// reads per K block for it. Here the weight rows are the UMMA M side (128 per tile) and the MN tokens
// (m rounded up to 16, 32 or 64) the UMMA N side, so a K block is one MN-column accumulator that
// each epilogue thread (one weight row) reads in a single tcgen05.ld.
//
// Roles (one CTA per SM, 192 threads):
//   warp 4      TMA producer: the 128x128 weight tile and the MN x 128 token tile (rows past m are
//               zero-filled by TMA) of each K block into an 8-stage ring.
//   warp 5      MMA issuer: per K block, 4 x tcgen05.mma.kind::i8 (M = 128, N = MN, K = 32) into one
//               of kTB TMEM accumulators.
//   warps 0-3   promotion epilogue: warp w owns TMEM lanes 32w..32w+31 (weight rows). The per-token
//               scales a_s[:, kb] * b_s[tile, kb] of 16 K blocks at a time are loaded with all loads
//               in flight (lane j: token j), staged in the warp's shared memory and read back as
//               broadcasts; the int32 partials are converted exactly and accumulated in fp32 with
//               packed FMAs.
//
// Schedule: stream-K over (tile, K block) units exactly as int8_gemm_kernel (Sched / SegIter): every
// CTA gets the same number of K blocks; partial tiles go through workspace slots of 128 x MN fp32
// (slot-major [token][row]) and the last contributor (one counter per tile and epilogue warp) sums
// them in ascending K order. Without a workspace: whole tiles per CTA.
#pragma once
#include "int8_gemm.cuh"

namespace dsv32 {
namespace gemm {

constexpr int kSwEpiWarps = 4;
constexpr int kSwThreads = (kSwEpiWarps + 2) * 32;
constexpr int kSwProducerWarp = kSwEpiWarps;
constexpr int kSwMmaWarp = kSwEpiWarps + 1;
constexpr int kSwMaxM = 64;  // largest m this path serves

constexpr int kSwScKb = 16;  // K blocks of token scales staged per warp at a time

// kPair = 2: a cluster of two CTAs per tile, each with half of the K blocks; the second pushes its fp32
// partial into the first's shared memory (kOffRecv, [MN][128] fp32) and arrives on the first's
// recv barrier of the same epilogue warp.
template <int MN, int kPair = 1>
struct SwapSmem {
  static_assert(MN == 16 || MN == 32 || MN == 64, "token tile of 16, 32 or 64 rows");
  static constexpr int kStages = (MN == 64 && kPair == 2) ? 6 : 8;
  static constexpr int kB = kBM * kBK;           // weight tile bytes (UMMA M side)
  static constexpr int kA = MN * kBK;            // token tile bytes (UMMA N side), a multiple of 1024
  static constexpr int kTB = 256 / MN > 8 ? 8 : 256 / MN;  // TMEM accumulators of MN columns
  static constexpr int kTmemCols = (MN * kTB < 32) ? 32 : MN * kTB;  // a power of two >= 32
  static constexpr int kOffB = 0;
  static constexpr int kOffA = kOffB + kStages * kB;
  static constexpr int kOffSc = kOffA + kStages * kA;  // per epilogue warp: kSwScKb x MN scales
  static constexpr int kOffRecv = kOffSc + kSwEpiWarps * kSwScKb * MN * 4;
  static constexpr int kOffBar = kOffRecv + (kPair == 2 ? kBM * MN * 4 : 0);
  // full[kStages], empty[kStages], tfull[kTB], tempty[kTB], mma_done, recv[kSwEpiWarps]
  static constexpr int kNumBars = 2 * kStages + 2 * kTB + 1 + kSwEpiWarps;
  static constexpr int kOffTmem = kOffBar + 8 * kNumBars;
  static constexpr int kOffAbort = kOffTmem + 4;
  static constexpr int kBytes = kOffAbort + 4;
  static constexpr int kAlloc = kBytes + 1024;
};

// Workspace for the swapped schedule: the counters of int8_gemm (first tiles x 4 of them used) and
// 2 * grid slots of 128 x MN fp32 after them.
__host__ __device__ inline int64_t swap_workspace_bytes(int mn, int grid, int64_t tiles_cap) {
  return counter_bytes(tiles_cap) + int64_t(2) * grid * kBM * mn * 4;
}

template <int MN>
DSV32_DEV void tmem_ld_mn(uint32_t taddr, uint32_t (&r)[MN]) {
  if constexpr (MN == 16) {
    tmem_ld16_async(taddr, r);
    tmem_wait_ld16(r);
  } else if constexpr (MN == 32) {
    tmem_ld32(taddr, r);
  } else {
    uint32_t(&lo)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
    uint32_t(&hi)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
    tmem_ld32_async(taddr, lo);
    tmem_ld32_async(taddr + 32, hi);
    tmem_wait_ld32(lo);
    tmem_wait_ld32(hi);
  }
}

// Stores row n's outputs C[j, n] for the tokens j < M (lanes hold consecutive n: coalesced per j).
template <int MN>
DSV32_DEV void store_col(const float (&acc)[MN], void* C, uint32_t out_kind, int M, int N, int n) {
#pragma unroll
  for (int j = 0; j < MN; ++j) {
    if (j < M) {
      const int64_t off = static_cast<int64_t>(j) * N + n;
      if (out_kind == kOutF32)
        static_cast<float*>(C)[off] = acc[j];
      else if (out_kind == kOutBF16)
        static_cast<__nv_bfloat16*>(C)[off] = __float2bfloat16_rn(acc[j]);
      else
        static_cast<__half*>(C)[off] = __float2half_rn(acc[j]);
    }
  }
}

// This CTA's segments: the stream-K / whole-tile schedule (SegIter), or with kPair = 2 the single
// segment of a CTA pair: tile blockIdx.x / 2, the first or second half of its K blocks by cluster rank
// (blockIdx.x % 2 for a 1-D grid of two-CTA clusters).
template <int kPair>
struct SwapIter {
  SegIter inner;
  bool used = false;
  DSV32_DEV SwapIter(const Sched& s) : inner(s) {}
  DSV32_DEV bool next(int& tile, int& kb0, int& kb1, bool& first) {
    if constexpr (kPair == 1) {
      return inner.next(tile, kb0, kb1, first);
    } else {
      if (used) return false;
      used = true;
      const int half = (inner.s.KG + 1) / 2;
      tile = blockIdx.x / 2;
      kb0 = (blockIdx.x & 1) ? half : 0;
      kb1 = (blockIdx.x & 1) ? inner.s.KG : half;
      first = true;
      return true;
    }
  }
};

template <int MN, bool kPartials, int kPair = 1>
__global__ void __launch_bounds__(kSwThreads, 1)
    int8_gemm_swap_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const float* __restrict__ a_s, const float* __restrict__ b_s, void* __restrict__ C,
                          uint32_t out_kind, int M, int N, int K, int32_t* __restrict__ partials,
                          uint8_t* __restrict__ workspace, int ws_tiles_cap) {
  using L = SwapSmem<MN, kPair>;
  constexpr int kStages = L::kStages;
  constexpr int kTB = L::kTB;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);

  const uint32_t sB = base + L::kOffB;
  const uint32_t sA = base + L::kOffA;
  const uint32_t bar0 = base + L::kOffBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto tfull_bar = [&](int b) { return bar0 + 8u * (2 * kStages + b); };
  auto tempty_bar = [&](int b) { return bar0 + 8u * (2 * kStages + kTB + b); };
  const uint32_t mma_done_bar = bar0 + 8u * (2 * kStages + 2 * kTB);
  auto recv_bar = [&](int w) { return bar0 + 8u * (2 * kStages + 2 * kTB + 1 + w); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffTmem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  Sched sch;
  sch.KG = K / kBK;
  sch.num_n = N / kBM;  // tiles: 128 weight rows each; a single token tile
  sch.num_tiles = sch.num_n;
  sch.grid = gridDim.x;
  sch.U = static_cast<long long>(sch.num_tiles) * sch.KG;
  sch.split = kPair == 1 && workspace != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < kTB; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), kSwEpiWarps);
    }
    mbar_init(mma_done_bar, 1);
    for (int w = 0; w < kSwEpiWarps; ++w) mbar_init(recv_bar(w), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kSwMmaWarp) tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if constexpr (kPair == 2) cluster_sync();  // the partner's barriers exist before any remote arrive
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // no global memory access before this point
  pdl_launch_dependents();

  if (warp == kSwProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      SwapIter<kPair> it(sch);
      int tile, kb0, kb1;
      bool first;
      while (ok && it.next(tile, kb0, kb1, first)) {
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, (KID_GEMM << 16) | 11)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), L::kB + L::kA);
          tma_load_2d(sB + stage * L::kB, &tmB, full_bar(stage), kb * kBK, tile * kBM);
          tma_load_2d(sA + stage * L::kA, &tmA, full_bar(stage), kb * kBK, 0);
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
  } else if (warp == kSwMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_i8(kBM, MN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t u = 0;  // K blocks multiplied by this CTA (selects the TMEM buffer)
      bool ok = true;
      SwapIter<kPair> it(sch);
      int tile, kb0, kb1;
      bool first;
      while (ok && it.next(tile, kb0, kb1, first)) {
        for (int kb = kb0; kb < kb1; ++kb, ++u) {
          const uint32_t buf = u % kTB;
          if (!mbar_wait(tempty_bar(buf), (u / kTB) & 1u, abort_flag, (KID_GEMM << 16) | 12) ||
              !mbar_wait(full_bar(stage), phase, abort_flag, (KID_GEMM << 16) | 13)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = sB + stage * L::kB;
          const uint32_t a_addr = sA + stage * L::kA;
          const uint32_t d_tmem = tmem_base + buf * MN;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            umma_i8(d_tmem, make_sdesc(b_addr + 32 * k, 128), make_sdesc(a_addr + 32 * k, 128), idesc,
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
  } else {
    // ------------------------------------------------------------ promotion epilogue (warps 0-3)
    const int r_local = warp * 32 + lane;  // weight row within the tile = TMEM lane
    const uint32_t t_lane = tmem_base + (uint32_t(warp * 32) << 16);
    float* sc_w = reinterpret_cast<float*>(smem + L::kOffSc) + warp * kSwScKb * MN;  // this warp's scales
    int* counters = reinterpret_cast<int*>(workspace);
    float* slots = workspace ? reinterpret_cast<float*>(workspace + counter_bytes(ws_tiles_cap)) : nullptr;
    constexpr int64_t kSlotFloats = static_cast<int64_t>(kBM) * MN;
    bool ok = true;
    __syncwarp();
    if (lane == 0) {
      for (int b = 0; b < kTB; ++b) mbar_arrive(tempty_bar(b));  // every accumulator starts free
    }
    uint32_t u = 0;
    SwapIter<kPair> it(sch);
    int tile, kb0, kb1;
    bool first_seg;
    while (ok && it.next(tile, kb0, kb1, first_seg)) {
      const int n = tile * kBM + r_local;  // N % 128 == 0: every row of a tile exists
      const float* bs_row = b_s + static_cast<int64_t>(tile) * sch.KG;
      float acc[MN];
#pragma unroll
      for (int j = 0; j < MN; ++j) acc[j] = 0.f;
      // token j's scale of K block kb (tokens past M read as 0)
      auto token_scale = [&](int kb, int j) {
        return j < M ? __ldg(a_s + static_cast<int64_t>(j) * sch.KG + kb) : 0.f;
      };
      for (int kb = kb0; kb < kb1; ++kb, ++u) {
        const uint32_t buf = u % kTB;
        const int ci = (kb - kb0) % kSwScKb;  // K block within the staged chunk
        if (ci == 0) {
          // Stage the per-token scales a_s[j, kb'] * b_s[tile, kb'] of the next kSwScKb K blocks (lane
          // j: tokens j and j + 32): every load of the chunk is in flight at once, one L2 round trip
          // per chunk instead of one per K block.
          const int nkb = min(kSwScKb, kb1 - kb);
          float bsv[kSwScKb], av0[kSwScKb], av1[kSwScKb];
#pragma unroll
          for (int i = 0; i < kSwScKb; ++i) {
            bsv[i] = i < nkb ? __ldg(bs_row + kb + i) : 0.f;
            av0[i] = i < nkb ? token_scale(kb + i, lane) : 0.f;
            av1[i] = (MN > 32 && i < nkb) ? token_scale(kb + i, lane + 32) : 0.f;
          }
          __syncwarp();  // the previous chunk's broadcasts are read
#pragma unroll
          for (int i = 0; i < kSwScKb; ++i) {
            if (lane < MN) sc_w[i * MN + lane] = av0[i] * bsv[i];
            if (MN > 32) sc_w[i * MN + lane + 32] = av1[i] * bsv[i];
          }
          __syncwarp();
        }
        if (!mbar_wait_warp(tfull_bar(buf), (u / kTB) & 1u, abort_flag, (KID_GEMM << 16) | 14)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[MN];
        tmem_ld_mn<MN>(t_lane + buf * MN, r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar(buf));  // the accumulator is in registers
        if constexpr (kPartials) {
#pragma unroll
          for (int j = 0; j < MN; ++j)
            if (j < M) partials[(static_cast<int64_t>(kb) * M + j) * N + n] = static_cast<int32_t>(r[j]);
        }
        const float4* sc4 = reinterpret_cast<const float4*>(sc_w + ci * MN);
#pragma unroll
        for (int j4 = 0; j4 < MN / 4; ++j4) {
          const float4 s4 = sc4[j4];  // same address across the warp: broadcast
          const float2 v0 = make_float2(static_cast<float>(static_cast<int32_t>(r[4 * j4])),
                                        static_cast<float>(static_cast<int32_t>(r[4 * j4 + 1])));
          const float2 v1 = make_float2(static_cast<float>(static_cast<int32_t>(r[4 * j4 + 2])),
                                        static_cast<float>(static_cast<int32_t>(r[4 * j4 + 3])));
          const float2 a0 = __ffma2_rn(v0, make_float2(s4.x, s4.y), make_float2(acc[4 * j4], acc[4 * j4 + 1]));
          const float2 a1 = __ffma2_rn(v1, make_float2(s4.z, s4.w), make_float2(acc[4 * j4 + 2], acc[4 * j4 + 3]));
          acc[4 * j4] = a0.x;
          acc[4 * j4 + 1] = a0.y;
          acc[4 * j4 + 2] = a1.x;
          acc[4 * j4 + 3] = a1.y;
        }
      }
      if (!ok) break;

      if constexpr (kPair == 2) {
        // CTA pair: the second CTA pushes this warp's 32 rows x MN partial (the second half of K) into
        // the first CTA's receive buffer and arrives on its barrier for this warp; the first adds it
        // to its own (first half + second half: deterministic) and stores.
        float* recv = reinterpret_cast<float*>(smem + L::kOffRecv);
        if (blockIdx.x & 1) {
          const uint32_t dst = cluster_map(smem_u32(recv), 0);
#pragma unroll
          for (int j = 0; j < MN; ++j) cluster_store(dst + 4u * static_cast<uint32_t>(j * kBM + r_local), acc[j]);
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(cluster_map(recv_bar(warp), 0));
        } else {
          if (!mbar_wait_cluster(recv_bar(warp), 0, abort_flag, (KID_GEMM << 16) | 15)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int j = 0; j < MN; ++j) acc[j] += recv[j * kBM + r_local];
          store_col<MN>(acc, C, out_kind, M, N, n);
        }
        continue;
      }
      if (kb0 == 0 && kb1 == sch.KG) {  // a whole tile: store directly
        store_col<MN>(acc, C, out_kind, M, N, n);
        continue;
      }
      // Partial tile: publish this warp's 32 rows x MN of the segment; the warp that completes this
      // sub-tile last (one counter per tile and warp) reduces and stores. Warp-local, as in
      // int8_gemm_kernel: no barrier across warps.
      const int slot = 2 * blockIdx.x + (first_seg ? 0 : 1);
      float* my_slot = slots + slot * kSlotFloats;
#pragma unroll
      for (int j = 0; j < MN; ++j) __stcg(my_slot + j * kBM + r_local, acc[j]);
      __threadfence();
      __syncwarp();
      const long long t_u0 = static_cast<long long>(tile) * sch.KG;
      const int c_first = sch.cta_of(t_u0);
      const int c_last = sch.cta_of(t_u0 + sch.KG - 1);
      int is_last = 0;
      if (lane == 0) {
        int* ctr = counters + static_cast<int64_t>(tile) * kSwEpiWarps + warp;
        const int prev = atomicAdd(ctr, 1);
        is_last = (prev == c_last - c_first);
        if (is_last) *ctr = 0;  // ready for the next launch
      }
      is_last = __shfl_sync(0xffffffffu, is_last, 0);
      if (!is_last) continue;
      __threadfence();
      // Every contributor has written its slot: sum them in ascending K order (deterministic).
#pragma unroll
      for (int j = 0; j < MN; ++j) acc[j] = 0.f;
      for (int cc = c_first; cc <= c_last; ++cc) {
        const int first_tile_of_cc = static_cast<int>(sch.ubeg(cc) / sch.KG);
        const int s = 2 * cc + (first_tile_of_cc == tile ? 0 : 1);
        const float* ps = slots + s * kSlotFloats;
#pragma unroll
        for (int j = 0; j < MN; ++j) acc[j] += __ldcg(ps + j * kBM + r_local);
      }
      store_col<MN>(acc, C, out_kind, M, N, n);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kSwMmaWarp) {
    __syncwarp();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
  // The first CTA of a pair stays until the second has finished writing into its shared memory (every
  // path of both CTAs reaches this point: all their waits are bounded).
  if constexpr (kPair == 2) cluster_sync();
}

}  // namespace gemm
}  // namespace dsv32
