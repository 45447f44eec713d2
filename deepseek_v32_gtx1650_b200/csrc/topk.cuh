// Per-row top-k selection over fp32 scores (the indexer's top-2048).
//
// The reference selects with torch.topk (test_kernels.py:125, bench_indexer_e2e.py:72-77)
// and compares sets tie-aware. This selection is deterministic: the k largest values,
// ties at the k-th value broken by lower position first; the output lists the selected
// positions in increasing position order, with their values. For a key range merged from
// shards, the candidate lists are concatenated in shard order and each is position-sorted,
// so "lower position" is "lower global key index", and the merge of per-shard top-k lists
// reproduces the single-GPU selection exactly.
//
// Values are mapped to order-preserving uint32 keys (larger float -> larger key, -inf is
// the smallest finite-or-masked key), so every comparison is an integer comparison.
//
// Two kernels:
//   topk_reg_kernel   rows of n <= THREADS*ITEMS: keys live in registers; the k-th key is found
//                     by a 32-step bisection over key bits (block-wide counts, no atomics).
//   topk_radix_kernel any n: three radix-histogram passes (11/11/10 bits) over the row in
//                     global memory (smem histogram), then the same ordered compaction.
#pragma once
#include "common.cuh"

namespace dsv32 {
namespace topk {

DSV32_DEV uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide sum; `scratch` holds 2 * (THREADS/32) ints and `parity` alternates between calls
// so one __syncthreads per call suffices.
template <int THREADS>
DSV32_DEV int block_sum(int v, int* scratch, int& parity) {
  constexpr int W = THREADS / 32;
  v = __reduce_add_sync(0xffffffffu, v);
  int* buf = scratch + parity * W;
  if ((threadIdx.x & 31) == 0) buf[threadIdx.x >> 5] = v;
  __syncthreads();
  int s = 0;
#pragma unroll
  for (int i = 0; i < W; ++i) s += buf[i];
  parity ^= 1;
  return s;
}

// Block-wide exclusive prefix sum in thread order.
template <int THREADS>
DSV32_DEV int block_excl_scan(int v, int* scratch, int& parity, int* total = nullptr) {
  constexpr int W = THREADS / 32;
  const int lane = threadIdx.x & 31;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  int* buf = scratch + parity * W;
  if (lane == 31) buf[threadIdx.x >> 5] = incl;
  __syncthreads();
  int before = 0, all = 0;
  const int wid = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const int t = buf[i];
    before += (i < wid) ? t : 0;
    all += t;
  }
  parity ^= 1;
  if (total) *total = all;
  return before + incl - v;
}

// Selected outputs of one thread's contiguous chunk, in position order.
template <int ITEMS>
DSV32_DEV void emit_chunk(const uint32_t (&key)[ITEMS], const float (&val)[ITEMS], int pos0, int n, uint32_t T,
                          int eq_before, int k_rem, int out_base, const int32_t* cand_row, long long idx_offset,
                          int32_t* out_idx_row, float* out_val_row) {
  int o = out_base;
  int eq = eq_before;
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int pos = pos0 + i;
    if (pos < n) {
      bool sel = key[i] > T;
      if (key[i] == T) {
        sel = eq < k_rem;
        ++eq;
      }
      if (sel) {
        out_idx_row[o] = cand_row ? cand_row[pos] : static_cast<int32_t>(pos + idx_offset);
        out_val_row[o] = val[i];
        ++o;
      }
    }
  }
}

template <int THREADS, int ITEMS>
__global__ void __launch_bounds__(THREADS) topk_reg_kernel(const float* __restrict__ vals, long long ld, int n,
                                                           const int32_t* __restrict__ cand_idx, long long cand_ld,
                                                           long long idx_offset, int k, int32_t* __restrict__ out_idx,
                                                           float* __restrict__ out_val) {
  __shared__ int scratch[2 * (THREADS / 32)];
  int parity = 0;
  const long long row = blockIdx.x;
  const float* v = vals + row * ld;
  const int pos0 = threadIdx.x * ITEMS;
  uint32_t key[ITEMS];
  float val[ITEMS];
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int pos = pos0 + i;
    val[i] = (pos < n) ? v[pos] : -INFINITY;
    key[i] = (pos < n) ? fkey(val[i]) : 0u;
  }
  int valid = 0;
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) valid += (pos0 + i < n) ? 1 : 0;

  // Largest T with count(key >= T) >= k, bit by bit from the top.
  uint32_t T = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = T | (1u << bit);
    int c = 0;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) c += (pos0 + i < n && key[i] >= cand) ? 1 : 0;
    if (block_sum<THREADS>(c, scratch, parity) >= k) T = cand;
  }
  int gt = 0, eq = 0;
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    if (pos0 + i < n) {
      gt += key[i] > T ? 1 : 0;
      eq += key[i] == T ? 1 : 0;
    }
  }
  (void)valid;
  const int G = block_sum<THREADS>(gt, scratch, parity);
  const int k_rem = k - G;  // ties at T to take, lowest positions first
  const int eq_before = block_excl_scan<THREADS>(eq, scratch, parity);
  const int take_eq = max(0, min(eq, k_rem - eq_before));
  const int out_base = block_excl_scan<THREADS>(gt + take_eq, scratch, parity);
  emit_chunk<ITEMS>(key, val, pos0, n, T, eq_before, k_rem, out_base, cand_idx ? cand_idx + row * cand_ld : nullptr,
                    idx_offset, out_idx + row * k, out_val + row * k);
}

// Generic version for long rows: radix histogram passes over global memory.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) topk_radix_kernel(const float* __restrict__ vals, long long ld, int n,
                                                             const int32_t* __restrict__ cand_idx, long long cand_ld,
                                                             long long idx_offset, int k, int32_t* __restrict__ out_idx,
                                                             float* __restrict__ out_val) {
  constexpr int kBins = 2048;
  __shared__ int hist[kBins];
  __shared__ int scratch[2 * (THREADS / 32)];
  __shared__ uint32_t s_prefix;
  __shared__ int s_krem;
  int parity = 0;
  const long long row = blockIdx.x;
  const float* v = vals + row * ld;

  uint32_t prefix = 0, pmask = 0;
  int k_rem = k;
  const int shifts[3] = {21, 10, 0};
  const int widths[3] = {11, 11, 10};
  for (int p = 0; p < 3; ++p) {
    const int nb = 1 << widths[p];
    for (int i = threadIdx.x; i < nb; i += THREADS) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += THREADS) {
      const uint32_t kk = fkey(v[i]);
      if ((kk & pmask) == prefix) atomicAdd(&hist[(kk >> shifts[p]) & (nb - 1)], 1);
    }
    __syncthreads();
    // Walk bins from the top: per-thread contiguous bin groups in descending order.
    constexpr int kPer = kBins / THREADS > 0 ? kBins / THREADS : 1;
    const int per = (nb + THREADS - 1) / THREADS;
    int local = 0;
    for (int j = 0; j < per; ++j) {
      const int bin = nb - 1 - (threadIdx.x * per + j);
      if (bin >= 0) local += hist[bin];
    }
    (void)kPer;
    const int before = block_excl_scan<THREADS>(local, scratch, parity);
    if (before < k_rem && k_rem <= before + local) {
      int acc = before;
      for (int j = 0; j < per; ++j) {
        const int bin = nb - 1 - (threadIdx.x * per + j);
        const int c = hist[bin];
        if (acc + c >= k_rem) {
          s_prefix = prefix | (uint32_t(bin) << shifts[p]);
          s_krem = k_rem - acc;
          break;
        }
        acc += c;
      }
    }
    __syncthreads();
    prefix = s_prefix;
    k_rem = s_krem;
    pmask |= uint32_t(nb - 1) << shifts[p];
    __syncthreads();
  }
  const uint32_t T = prefix;
  // Ordered compaction over per-thread contiguous chunks.
  const int chunk = (n + THREADS - 1) / THREADS;
  const int p0 = threadIdx.x * chunk;
  const int p1 = min(n, p0 + chunk);
  int gt = 0, eq = 0;
  for (int pos = p0; pos < p1; ++pos) {
    const uint32_t kk = fkey(v[pos]);
    gt += kk > T;
    eq += kk == T;
  }
  const int eq_before = block_excl_scan<THREADS>(eq, scratch, parity);
  const int take_eq = max(0, min(eq, k_rem - eq_before));
  int o = block_excl_scan<THREADS>(gt + take_eq, scratch, parity);
  const int32_t* cand_row = cand_idx ? cand_idx + row * cand_ld : nullptr;
  int32_t* oi = out_idx + row * k;
  float* ov = out_val + row * k;
  int e = eq_before;
  for (int pos = p0; pos < p1; ++pos) {
    const float x = v[pos];
    const uint32_t kk = fkey(x);
    bool sel = kk > T;
    if (kk == T) {
      sel = e < k_rem;
      ++e;
    }
    if (sel) {
      oi[o] = cand_row ? cand_row[pos] : static_cast<int32_t>(pos + idx_offset);
      ov[o] = x;
      ++o;
    }
  }
}

}  // namespace topk
}  // namespace dsv32
