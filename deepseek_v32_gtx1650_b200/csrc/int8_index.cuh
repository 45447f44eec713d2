// int8_index: DeepSeek-V3.2 lightning indexer on the sm_100a tensor cores.
//
//   score[b, m, n] = k_s[b, n] * sum_h w[b, m, h] * relu( sum_d q[b, m, h, d] * k[b, n, d] )
//   causal: score = -inf where n > start + m
//
// Semantics: reference.py:27-34 (int8_index_ref) and kernels.py:134-162. Operands keep the
// reference layout: q [B, M, H, D] int8, k [B, N, D] int8, w [B, M, H] fp32, k_s [B, N] fp32,
// out [B, M, N] fp32.
//
// Mapping: UMMA M = 128 keys (TMEM lanes), UMMA N = QB*H (query, head) pairs (QB*H = 256), K = D.
// A work unit is (batch, block of QB queries, chunk of 128-key tiles). The kernel is persistent:
// one CTA per SM walks its units (heaviest causal query blocks first, dealt out in snake order so
// every SM gets about the same number of tiles) and keeps its TMEM, barriers and pipelines across
// units, so consecutive units overlap (the next unit's Q and key tiles load while the current
// one is still in the epilogue).
//   warps 0-15  epilogue: each thread owns one key and reduces relu(logit) * w over the heads of
//               its queries entirely in registers (no cross-lane reduction), then scales by k_s and
//               stores. Two groups of eight warps take alternate key tiles (group g reads TMEM buffer
//               g), so one group computes while the other waits for its accumulator; in a group, warp
//               w reads TMEM lanes 32*(w%4).. and column half (w/4)%2 (QB/2 queries) in two passes.
//   warp 16     TMA producer: the unit's Q block into one of two Q buffers, then its key tiles
//               into a 4-stage ring.
//   warp 17     MMA issuer: D / 32 MMAs per key tile into one of two int32 TMEM accumulators.
//   warp 18     writes -inf for the key tiles that no query of a unit can see (causal), which are
//               neither loaded nor multiplied (the reference's tile skip, kernels.py:145-148). With
//               fill_masked == 0 (scores used only as the selection's scratch, whose causal rows are
//               never read past their visible length) those tiles are left unwritten.
// Selected rows (kSel; the fused indexer + top-k of one causal batch): rows m < m_triv see at most
// sel_k keys, so their top-sel_k is their first sel_k positions in order. The epilogue writes their
// visible scores and ids straight to the selection outputs and the -inf writer their masked ones;
// their score rows are written only with fill_masked (scores kept as output).
// Keys and their scales of batch b start at key b * ks_ld (ks_ld >= N: a cache with spare capacity
// is read in place).
//
// Per logit: relu and the int32 -> fp32 conversion in one saturating fp32 multiply of the raw bits
// (relu_i32_x2m22, exact for |logit| <= D*128*128 <= 2^21, giving relu * 2^-22), then one fused
// multiply-add with the head weight (packed f32x2); the 2^-22 is folded into k_s. Everything runs on
// the FP32 pipe; the results equal relu-then-convert bit for bit (power-of-two scalings, no
// subnormal intermediates for any realistic head weight).
// The first MMA of each key tile overwrites the accumulator, so buffers need no clearing.
#pragma once
#include "common.cuh"

namespace dsv32 {
namespace index {

constexpr int kKeysPerTile = 128;
constexpr int kStages = 4;
constexpr int kEpiWarps = 16;
constexpr int kThreads = (kEpiWarps + 3) * 32;  // + producer, MMA and one -inf writer warp
// 608 threads x 104 registers = 63232 of the SM's 65536; no register re-balancing (the warps do
// not form whole warpgroups past the epilogue, and 104 is what the epilogue needs).
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;
constexpr int kFillWarp = kEpiWarps + 2;
constexpr int kNmma = 256;  // QB * H

template <int H, int D>
struct Cfg {
  static constexpr int QB = kNmma / H;                 // queries per block
  static constexpr int kQBytes = QB * H * D;           // Q tile bytes
  static constexpr int kKBytes = kKeysPerTile * D;     // key tile bytes per stage
  static constexpr int kColsPerWarp = kNmma / 2;      // columns per epilogue warp (one half)
  static constexpr int kQPerWarp = QB / 2;            // queries per epilogue warp
  static constexpr int kQPerPass = kQPerWarp / 2;     // queries per 64-column pass of a warp
  static constexpr int kOffQ = 0;                      // two Q buffers
  static constexpr int kOffK = kOffQ + 2 * kQBytes;
  static constexpr int kOffW = kOffK + kStages * kKBytes;  // per epilogue warp: two units' weights
  static constexpr int kOffBar = kOffW + kEpiWarps * 2 * kColsPerWarp * 4;
  static_assert(kColsPerWarp == 32 * 4, "one 16-byte copy per lane per unit's weights");
  // qfull[2], qempty[2], kfull[kStages], kempty[kStages], tfull[2], tempty[2], mma_done
  static constexpr int kNumBars = 9 + 2 * kStages;
  static constexpr int kOffTmem = kOffBar + 8 * kNumBars;
  static constexpr int kOffAbort = kOffTmem + 4;
  static constexpr int kBytes = kOffAbort + 4;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(QB * H == kNmma, "QB*H must be 256");
  static_assert(D == 64 || D == 128, "head dim must be 64 or 128");
  static_assert(QB % 4 == 0, "four query quarters");
};

DSV32_DEV void drain_wait(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > DSV32_WAIT_LIMIT_CYCLES / 16) break;
  }
}

struct Unit {
  int b, m0, kt0, kt_vis, kt1;
};

// Work unit number `idx`. Units are numbered so that the heaviest causal query blocks come first.
DSV32_DEV Unit decode_unit(int idx, int M, int N, int QB, int causal, long long start, int tiles_per_chunk,
                           int num_chunks) {
  const int NQB = (M + QB - 1) / QB;
  const int NT = (N + kKeysPerTile - 1) / kKeysPerTile;
  const int c = idx % num_chunks;
  const int rest = idx / num_chunks;
  int qb = rest % NQB;
  if (causal) qb = NQB - 1 - qb;
  Unit u;
  u.b = rest / NQB;
  u.m0 = qb * QB;
  u.kt0 = c * tiles_per_chunk;
  u.kt1 = min(NT, u.kt0 + tiles_per_chunk);
  u.kt_vis = u.kt1;
  if (causal) {
    const long long m_last = min(M - 1, u.m0 + QB - 1);
    const long long lim = start + m_last + 1;  // keys [0, lim) are visible to some query
    const long long vis_tiles = lim <= 0 ? 0 : (lim + kKeysPerTile - 1) / kKeysPerTile;
    u.kt_vis = static_cast<int>(max(static_cast<long long>(u.kt0), min(static_cast<long long>(u.kt1), vis_tiles)));
  }
  return u;
}

// The r-th unit of this CTA in snake order (round r covers units [r*G, (r+1)*G); odd rounds run
// backwards), or -1 past the end.
DSV32_DEV int unit_of_round(int r, int units) {
  const int G = static_cast<int>(gridDim.x);
  const long long idx = static_cast<long long>(r) * G + ((r & 1) ? (G - 1 - static_cast<int>(blockIdx.x))
                                                                 : static_cast<int>(blockIdx.x));
  return idx < units ? static_cast<int>(idx) : -1;
}

// kSel: the launch selects the leading rows itself (m_triv > 0); kept out of the plain instantiation,
// whose epilogue loop it would otherwise lengthen.
template <int H, int D, bool kSel>
__global__ void __launch_bounds__(kThreads, 1)
    int8_index_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const float* __restrict__ w, const float* __restrict__ k_s, float* __restrict__ out, int M,
                      int N, int causal, long long start, int tiles_per_chunk, int num_chunks, int units,
                      long long ks_ld, int fill_masked, int32_t* __restrict__ sel_idx,
                      float* __restrict__ sel_val, int sel_k, int m_triv, int key_offset) {
  using C = Cfg<H, D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);

  const uint32_t sQ = base + C::kOffQ;
  const uint32_t sK = base + C::kOffK;
  const uint32_t bar0 = base + C::kOffBar;
  auto qfull_bar = [&](int b) { return bar0 + 8u * b; };
  auto qempty_bar = [&](int b) { return bar0 + 8u * (2 + b); };
  auto kfull_bar = [&](int s) { return bar0 + 8u * (4 + s); };
  auto kempty_bar = [&](int s) { return bar0 + 8u * (4 + kStages + s); };
  auto tfull_bar = [&](int b) { return bar0 + 8u * (4 + 2 * kStages + b); };
  auto tempty_bar = [&](int b) { return bar0 + 8u * (6 + 2 * kStages + b); };
  const uint32_t mma_done_bar = bar0 + 8u * (8 + 2 * kStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffAbort);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(qfull_bar(b), 1);
      mbar_init(qempty_bar(b), 1);
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), kEpiWarps / 2);  // the epilogue group that reads buffer b
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(kfull_bar(s), 1);
      mbar_init(kempty_bar(s), 1);
    }
    mbar_init(mma_done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tmem_alloc(smem_u32(tmem_slot), 2 * kNmma);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // no global memory access before this point
  pdl_launch_dependents();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      int stage = 0;
      uint32_t phase = 0;
      int k_issued = 0, q_issued = 0;
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int idx = unit_of_round(r, units);
        if (idx < 0) break;
        const Unit un = decode_unit(idx, M, N, C::QB, causal, start, tiles_per_chunk, num_chunks);
        if (un.kt_vis == un.kt0) continue;  // nothing to multiply
        const int qb = q_issued & 1;
        if (!mbar_wait(qempty_bar(qb), ((q_issued >> 1) & 1) ^ 1u, abort_flag, (KID_INDEX << 16) | 6)) break;
        mbar_arrive_expect_tx(qfull_bar(qb), C::kQBytes);
        tma_load_3d(sQ + qb * C::kQBytes, &tmQ, qfull_bar(qb), 0, un.m0 * H, un.b);
        ++q_issued;
        for (int kt = un.kt0; kt < un.kt_vis; ++kt) {
          if (!mbar_wait(kempty_bar(stage), phase ^ 1u, abort_flag, (KID_INDEX << 16) | 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(kfull_bar(stage), C::kKBytes);
          tma_load_3d(sK + stage * C::kKBytes, &tmK, kfull_bar(stage), 0, kt * kKeysPerTile, un.b);
          ++k_issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Wait for the last loads issued into every buffer to land before the CTA can exit.
      for (int i = 0; i < kStages && i < k_issued; ++i) {
        if (--stage < 0) {
          stage = kStages - 1;
          phase ^= 1u;
        }
        drain_wait(kfull_bar(stage), phase);
      }
      for (int j = max(0, q_issued - 2); j < q_issued; ++j) drain_wait(qfull_bar(j & 1), (j >> 1) & 1);
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_i8(kKeysPerTile, kNmma);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t i = 0;  // key tiles multiplied by this CTA (selects the TMEM buffer)
      int j = 0;       // units multiplied by this CTA (selects the Q buffer)
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int idx = unit_of_round(r, units);
        if (idx < 0) break;
        const Unit un = decode_unit(idx, M, N, C::QB, causal, start, tiles_per_chunk, num_chunks);
        if (un.kt_vis == un.kt0) continue;
        const int qb = j & 1;
        if (!mbar_wait(qfull_bar(qb), (j >> 1) & 1, abort_flag, (KID_INDEX << 16) | 2)) break;
        const uint32_t q_addr = sQ + qb * C::kQBytes;
        for (int kt = un.kt0; kt < un.kt_vis; ++kt, ++i) {
          const uint32_t buf = i & 1u;
          if (!mbar_wait(tempty_bar(buf), (i >> 1) & 1u, abort_flag, (KID_INDEX << 16) | 3) ||
              !mbar_wait(kfull_bar(stage), phase, abort_flag, (KID_INDEX << 16) | 4)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = sK + stage * C::kKBytes;
          const uint32_t d_tmem = tmem_base + buf * kNmma;
#pragma unroll
          for (int k = 0; k < D / 32; ++k) {
            umma_i8(d_tmem, make_sdesc(k_addr + 32 * k, D), make_sdesc(q_addr + 32 * k, D), idesc, k > 0 ? 1u : 0u);
          }
          umma_commit(kempty_bar(stage));
          umma_commit(tfull_bar(buf));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma_commit(qempty_bar(qb));  // the Q buffer is free once this unit's MMAs are done
        ++j;
      }
      umma_commit(mma_done_bar);
      drain_wait(mma_done_bar, 0);
    }
  } else if (warp == kFillWarp) {
    // ------------------------------------------------------------ -inf for invisible key tiles
    const int ft = lane;
    const bool vec4 = (N % 4) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
    for (int r = 0; fill_masked || kSel; ++r) {
      const int idx = unit_of_round(r, units);
      if (idx < 0) break;
      const Unit un = decode_unit(idx, M, N, C::QB, causal, start, tiles_per_chunk, num_chunks);
      if (un.kt_vis == un.kt1) continue;
      const int n_lo = un.kt_vis * kKeysPerTile;
      const int n_hi = min(N, un.kt1 * kKeysPerTile);
      float* out_b = out + static_cast<int64_t>(un.b) * M * N;
      for (int q = 0; q < C::QB; ++q) {
        const int m = un.m0 + q;
        if (m >= M) break;
        if (fill_masked) {
          float* row = out_b + static_cast<int64_t>(m) * N;
          if (vec4) {  // n_lo is a multiple of 128 and rows are 16-byte aligned
            float4* row4 = reinterpret_cast<float4*>(row);
            const float4 ninf4 = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            for (int n4 = n_lo / 4 + ft; n4 < n_hi / 4; n4 += 32) row4[n4] = ninf4;
            for (int n = (n_hi & ~3) + ft; n < n_hi; n += 32) row[n] = -INFINITY;
          } else {
            for (int n = n_lo + ft; n < n_hi; n += 32) row[n] = -INFINITY;
          }
        }
        if (kSel && m < m_triv) {  // a row selected here: its masked positions below sel_k
          const int64_t so = (static_cast<int64_t>(un.b) * M + m) * sel_k;
          for (int n = n_lo + ft; n < min(n_hi, sel_k); n += 32) {
            sel_val[so + n] = -INFINITY;
            sel_idx[so + n] = n + key_offset;
          }
        }
      }
    }
  } else if (warp < kEpiWarps) {
    // ------------------------------------------------------------ epilogue (two groups of 8 warps)
    // Group g reads TMEM buffer g, i.e. the key tiles i (counted over all units of this CTA) with
    // i % 2 == g; while one group waits for its next accumulator the other computes. In a group, warp
    // (wq, ch) reads lane quarter wq (keys) and column half ch (QB / 2 queries) in two passes of 64
    // columns, releasing the buffer after the second pass's TMEM read.
    const int g = warp >> 3;
    const int wq = warp & 3;   // TMEM lane quarter (keys); a warp reads lanes 32 * (warp % 4) ..
    const int ch = (warp >> 2) & 1;
    const int q_first = ch * C::kQPerWarp;  // first query (within the block) of this warp
    const uint32_t t_lane = tmem_base + (uint32_t(wq * 32) << 16) + uint32_t(g * kNmma + ch * C::kColsPerWarp);
    float* sWw = reinterpret_cast<float*>(smem + C::kOffW) + warp * 2 * C::kColsPerWarp;  // this warp's
    const float4* w4p = reinterpret_cast<const float4*>(sWw);  // the half the tile loop reads
    bool ok = true;
    __syncwarp();  // this group's accumulator starts free
    if (lane == 0) mbar_arrive(tempty_bar(g));
    const int n_base = wq * 32 + lane;
    // Head weights of this warp's queries in the unit of round rr (its QB / 2 rows of w, contiguous;
    // rows past M zero-filled) into the staging half of the warp's private copy, one unit ahead, as
    // asynchronous copies (one 16-byte copy per lane, no registers held while in flight): their
    // latency falls inside the previous unit. At a unit's start each lane moves its 16 bytes to the
    // half the tile loop reads, which keeps that loop's addresses fixed. (Weights loaded into
    // registers a unit ahead instead cost the long-row loop 8 %; reading the two halves
    // alternately, 3 %.)
    auto fetch_w = [&](int rr) {
      const int idx = unit_of_round(rr, units);
      if (idx < 0) return;
      const Unit u = decode_unit(idx, M, N, C::QB, causal, start, tiles_per_chunk, num_chunks);
      const int e = lane * 4;
      const int m = u.m0 + q_first + e / H;
      const float* src = (m < M) ? w + (static_cast<int64_t>(u.b) * M + m) * H + (e % H) : w;
      cp_async16(smem_u32(sWw + C::kColsPerWarp + e), src, m < M ? 16u : 0u);
      cp_async_commit();
    };
    fetch_w(0);
    uint32_t i = 0;  // key tiles of all units so far (both groups)
    for (int r = 0; ok; ++r) {
      const int idx = unit_of_round(r, units);
      if (idx < 0) break;
      // Round r's weights have landed in the staging half: each lane moves its own 16 bytes (its
      // copies are complete once it has waited), the warp barrier orders round r - 1's reads of the
      // loop half before, and every lane's move before round r's reads and the next copy.
      cp_async_wait_all();
      __syncwarp();
      reinterpret_cast<float4*>(sWw)[lane] = reinterpret_cast<const float4*>(sWw + C::kColsPerWarp)[lane];
      __syncwarp();
      fetch_w(r + 1);
      const Unit un = decode_unit(idx, M, N, C::QB, causal, start, tiles_per_chunk, num_chunks);
      if (un.kt_vis == un.kt0) continue;
      const uint32_t i0 = i;
      i += static_cast<uint32_t>(un.kt_vis - un.kt0);
      const int kt_first = un.kt0 + static_cast<int>((static_cast<uint32_t>(g) - i0) & 1u);
      if (kt_first >= un.kt_vis) continue;  // the unit's only tile is the other group's
      uint32_t kk = (i0 + (g == 0 ? 1u : 0u)) >> 1;  // this group's tiles before this unit
      // Per unit: this thread's key column and its k_s, the first query's output row and, for
      // causal rows, the last visible tile offset of the first query (query q: lim0 + q).
      const int m_first = un.m0 + q_first;
      const float* ksp = k_s + static_cast<int64_t>(un.b) * ks_ld + n_base;
      float* out0 = out + (static_cast<int64_t>(un.b) * M + m_first) * N + n_base;
      const long long l0 = causal ? start + m_first - n_base : (1LL << 30);
      const int lim0 = static_cast<int>(l0 < -(1LL << 30) ? -(1LL << 30) : (l0 > (1LL << 30) ? (1LL << 30) : l0));
      // Rows selected here (m < m_triv: at most sel_k visible keys) have their scores written only
      // when kept as output. sel_unit (warp-uniform): some query of this warp is such a row.
      const bool sel_unit = kSel && m_first < m_triv;
      // k_s of this thread's key in this group's next tile, loaded a tile ahead.
      float ks_next = (kt_first * kKeysPerTile + n_base < N) ? __ldg(ksp + kt_first * kKeysPerTile) : 0.f;
      for (int kt = kt_first; kt < un.kt_vis; kt += 2, ++kk) {
        const int toff = kt * kKeysPerTile;
        const bool n_ok = toff + n_base < N;
        // k_s * 2^22 undoes the 2^-22 of the relu step (power-of-two scalings: same rounding).
        const float ks = ks_next * 0x1p22f;
        ks_next = (kt + 2 < un.kt_vis && toff + 2 * kKeysPerTile + n_base < N) ? __ldg(ksp + toff + 2 * kKeysPerTile)
                                                                               : 0.f;
        if (!mbar_wait_warp(tfull_bar(g), kk & 1u, abort_flag, (KID_INDEX << 16) | 5)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
          // Both 32-column chunks of this pass in flight at once, then one wait.
          uint32_t ra[32], rb[32];
          tmem_ld32_async(t_lane + pass * 64, ra);
          tmem_ld32_async(t_lane + pass * 64 + 32, rb);
          tmem_wait_ld32(ra);
          tmem_wait_ld32(rb);
          if (pass == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(g));  // the accumulator is in registers now
          }
          // Two accumulators per query (even / odd column pairs) halve the FMA dependency chain.
          float2 acc[C::kQPerPass][2];
#pragma unroll
          for (int q = 0; q < C::kQPerPass; ++q) acc[q][0] = acc[q][1] = make_float2(0.f, 0.f);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t(&rr)[32] = c ? rb : ra;
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 w4 = w4p[pass * 16 + c * 8 + j4];  // same address across the warp: broadcast
              const int q = (c * 32 + 4 * j4) / H;             // query of these 4 columns in the pass
              const float2 v0 = make_float2(relu_i32_x2m22(rr[4 * j4]), relu_i32_x2m22(rr[4 * j4 + 1]));
              const float2 v1 = make_float2(relu_i32_x2m22(rr[4 * j4 + 2]), relu_i32_x2m22(rr[4 * j4 + 3]));
              acc[q][0] = __ffma2_rn(v0, make_float2(w4.x, w4.y), acc[q][0]);
              acc[q][1] = __ffma2_rn(v1, make_float2(w4.z, w4.w), acc[q][1]);
            }
          }
          if (n_ok) {
#pragma unroll
            for (int q = 0; q < C::kQPerPass; ++q) {
              const int qw = pass * C::kQPerPass + q;  // query within the warp
              const int m = m_first + qw;
              float sc = ((acc[q][0].x + acc[q][0].y) + (acc[q][1].x + acc[q][1].y)) * ks;
              if (toff > lim0 + qw) sc = -INFINITY;
              if (!sel_unit) {
                if (m < M) out0[static_cast<int64_t>(qw) * N + toff] = sc;
              } else if (kSel) {
                if (m < M && (fill_masked || m >= m_triv)) out0[static_cast<int64_t>(qw) * N + toff] = sc;
                if (m < m_triv && toff + n_base < sel_k) {  // output j of such a row is position j
                  const int64_t so = (static_cast<int64_t>(un.b) * M + m) * sel_k + toff + n_base;
                  sel_val[so] = sc;
                  sel_idx[so] = toff + n_base + key_offset;
                }
              }
            }
          }
        }
      }
    }
    cp_async_wait_all();  // a weight copy issued before an abort lands before the CTA can exit
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    __syncwarp();
    tmem_dealloc(tmem_base, 2 * kNmma);
  }
}

}  // namespace index
}  // namespace dsv32
