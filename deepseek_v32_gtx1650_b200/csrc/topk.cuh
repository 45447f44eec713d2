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
// Algorithm (radix select on order-preserving uint32 keys; larger float -> larger key):
//  1. Block reductions give the number of finite values and the min / max finite key. Masked
//     (-inf) scores never enter a histogram: when at most k values are finite, the threshold is
//     the -inf key itself and the lowest-position masked keys fill the list.
//  2. Otherwise the bits above the highest bit in which min and max differ are common to every
//     finite key; the remaining bits are resolved with 11-bit shared-memory histograms (at most
//     three passes), each pass counting only keys that match the prefix found so far.
//  3. Ordered compaction: block-wide prefix sums over per-thread contiguous chunks place every
//     key > T and the first k_rem keys == T in position order.
// topk_reg_kernel keeps a row of up to THREADS*ITEMS keys in registers (one read of the row);
// topk_gmem_kernel re-reads longer rows from global memory (L2) in each pass.
#pragma once
#include "common.cuh"

namespace dsv32 {
namespace topk {

constexpr uint32_t kNegInfKey = 0x007FFFFFu;  // key of -inf: below every finite value
constexpr int kHistBits = 11;

DSV32_DEV uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

DSV32_DEV float fkey_inv(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

// Keys of a row fall into: "above" (> the -inf key: finite, +inf, +NaN), the -inf key, and
// below it (negative NaN). Masked -inf entries are counted, never histogrammed.
DSV32_DEV bool prefix_match(uint32_t key, uint32_t prefix, int shift) {
  return shift >= 32 || (key >> shift) == (prefix >> shift);
}

// Block-wide sum / min / max; `scratch` holds 2 * 32 ints and `parity` alternates so one
// __syncthreads per call suffices.
template <int THREADS>
DSV32_DEV int block_sum(int v, int* scratch, int& parity) {
  constexpr int W = THREADS / 32;
  v = __reduce_add_sync(0xffffffffu, v);
  int* buf = scratch + parity * 32;
  if ((threadIdx.x & 31) == 0) buf[threadIdx.x >> 5] = v;
  __syncthreads();
  int s = 0;
#pragma unroll
  for (int i = 0; i < W; ++i) s += buf[i];
  parity ^= 1;
  return s;
}

template <int THREADS>
DSV32_DEV void block_minmax(uint32_t& mn, uint32_t& mx, uint32_t* scratch, int& parity) {
  constexpr int W = THREADS / 32;
  mn = __reduce_min_sync(0xffffffffu, mn);
  mx = __reduce_max_sync(0xffffffffu, mx);
  uint32_t* buf = scratch + parity * 64;
  if ((threadIdx.x & 31) == 0) {
    buf[threadIdx.x >> 5] = mn;
    buf[32 + (threadIdx.x >> 5)] = mx;
  }
  __syncthreads();
  mn = 0xFFFFFFFFu;
  mx = 0u;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    mn = min(mn, buf[i]);
    mx = max(mx, buf[32 + i]);
  }
  parity ^= 1;
}

// Block-wide exclusive prefix sum in thread order.
template <int THREADS>
DSV32_DEV int block_excl_scan(int v, int* scratch, int& parity) {
  constexpr int W = THREADS / 32;
  const int lane = threadIdx.x & 31;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  int* buf = scratch + parity * 32;
  if (lane == 31) buf[threadIdx.x >> 5] = incl;
  __syncthreads();
  int before = 0;
  const int wid = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < W; ++i) before += (i < wid) ? buf[i] : 0;
  parity ^= 1;
  return before + incl - v;
}

// Shared state of one selection.
struct SelShared {
  int hist[1 << kHistBits];
  int scratch[64];
  uint32_t mm[128];
  uint32_t prefix;
  int krem;
};

// After a histogram over digit bits [shift, shift + d), find the digit of the k_rem-th largest
// participating key. Updates prefix / k_rem in shared memory (all threads read them after).
template <int THREADS>
DSV32_DEV void pick_digit(SelShared& sh, int nbins, int shift, uint32_t prefix, int k_rem, int& parity) {
  const int per = (nbins + THREADS - 1) / THREADS;  // bins per thread, descending order
  int local = 0;
  for (int j = 0; j < per; ++j) {
    const int bin = nbins - 1 - (threadIdx.x * per + j);
    if (bin >= 0) local += sh.hist[bin];
  }
  const int before = block_excl_scan<THREADS>(local, sh.scratch, parity);
  if (before < k_rem && k_rem <= before + local) {
    int acc = before;
    for (int j = 0; j < per; ++j) {
      const int bin = nbins - 1 - (threadIdx.x * per + j);
      const int c = sh.hist[bin];
      if (acc + c >= k_rem) {
        sh.prefix = prefix | (uint32_t(bin) << shift);
        sh.krem = k_rem - acc;
        break;
      }
      acc += c;
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------- register rows
template <int THREADS, int ITEMS>
__global__ void __launch_bounds__(THREADS) topk_reg_kernel(const float* __restrict__ vals, long long ld, int n,
                                                           const int32_t* __restrict__ cand_idx, long long cand_ld,
                                                           long long idx_offset, int k, int32_t* __restrict__ out_idx,
                                                           float* __restrict__ out_val) {
  __shared__ SelShared sh;
  int parity = 0;
  const long long row = blockIdx.x;
  const float* v = vals + row * ld;
  const int pos0 = threadIdx.x * ITEMS;
  uint32_t key[ITEMS];
  // Each thread owns ITEMS consecutive positions (position order = thread order).
  if ((ld & 3) == 0 && (reinterpret_cast<uintptr_t>(vals) & 15u) == 0 && (ITEMS % 4) == 0 && pos0 + ITEMS <= n) {
#pragma unroll
    for (int i = 0; i < ITEMS; i += 4) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(v + pos0 + i));
      key[i] = fkey(f.x);
      key[i + 1] = fkey(f.y);
      key[i + 2] = fkey(f.z);
      key[i + 3] = fkey(f.w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) key[i] = (pos0 + i < n) ? fkey(__ldg(v + pos0 + i)) : 0u;
  }
  // 1. counts above / at the -inf key; range of the keys that take part in the histograms
  int n_above = 0, n_ninf = 0;
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const bool valid = pos0 + i < n;
    n_above += (valid && key[i] > kNegInfKey) ? 1 : 0;
    n_ninf += (valid && key[i] == kNegInfKey) ? 1 : 0;
  }
  const int above = block_sum<THREADS>(n_above, sh.scratch, parity);
  const int ninf = block_sum<THREADS>(n_ninf, sh.scratch, parity);
  uint32_t T;
  int k_rem;
  if (above < k && above + ninf >= k) {
    T = kNegInfKey;  // all values above -inf, then the lowest-position -inf entries
    k_rem = k - above;
  } else {
    // 2. radix select among keys >= floor (above -inf; or every key if negative NaNs are needed)
    const uint32_t floor_key = (above >= k) ? kNegInfKey + 1u : 0u;
    uint32_t mn = 0xFFFFFFFFu, mx = 0u;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const bool part = pos0 + i < n && key[i] >= floor_key;
      mn = part ? min(mn, key[i]) : mn;
      mx = part ? max(mx, key[i]) : mx;
    }
    block_minmax<THREADS>(mn, mx, sh.mm, parity);
    int shift = (mn == mx) ? 0 : 32 - __clz(mn ^ mx);  // bits [shift, 32) common to every participant
    uint32_t prefix = (shift >= 32) ? 0u : (mx & ~((1u << shift) - 1u));
    k_rem = k;
    while (shift > 0) {
      const int d = min(kHistBits, shift);
      const int nbins = 1 << d;
      for (int i = threadIdx.x; i < nbins; i += THREADS) sh.hist[i] = 0;
      __syncthreads();
      const int ns = shift - d;
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        const bool part = pos0 + i < n && key[i] >= floor_key && prefix_match(key[i], prefix, shift);
        if (part) atomicAdd(&sh.hist[(key[i] >> ns) & (nbins - 1)], 1);
      }
      __syncthreads();
      pick_digit<THREADS>(sh, nbins, ns, prefix, k_rem, parity);
      prefix = sh.prefix;
      k_rem = sh.krem;
      shift = ns;
      __syncthreads();
    }
    T = prefix;
  }
  // 3. ordered compaction
  int gt = 0, eq = 0;
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    if (pos0 + i < n) {
      gt += key[i] > T ? 1 : 0;
      eq += key[i] == T ? 1 : 0;
    }
  }
  const int eq_before = block_excl_scan<THREADS>(eq, sh.scratch, parity);
  const int take_eq = max(0, min(eq, k_rem - eq_before));
  int o = block_excl_scan<THREADS>(gt + take_eq, sh.scratch, parity);
  const int32_t* cand_row = cand_idx ? cand_idx + row * cand_ld : nullptr;
  int32_t* oi = out_idx + row * k;
  float* ov = out_val + row * k;
  int e = eq_before;
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int pos = pos0 + i;
    if (pos < n) {
      bool sel = key[i] > T;
      if (key[i] == T) {
        sel = e < k_rem;
        ++e;
      }
      if (sel) {
        oi[o] = cand_row ? cand_row[pos] : static_cast<int32_t>(pos + idx_offset);
        ov[o] = fkey_inv(key[i]);
        ++o;
      }
    }
  }
}

// ---------------------------------------------------------------------------- long rows
template <int THREADS>
__global__ void __launch_bounds__(THREADS) topk_gmem_kernel(const float* __restrict__ vals, long long ld, int n,
                                                            const int32_t* __restrict__ cand_idx, long long cand_ld,
                                                            long long idx_offset, int k, int32_t* __restrict__ out_idx,
                                                            float* __restrict__ out_val) {
  __shared__ SelShared sh;
  int parity = 0;
  const long long row = blockIdx.x;
  const float* v = vals + row * ld;
  int n_above = 0, n_ninf = 0;
  for (int i = threadIdx.x; i < n; i += THREADS) {
    const uint32_t kk = fkey(__ldg(v + i));
    n_above += kk > kNegInfKey ? 1 : 0;
    n_ninf += kk == kNegInfKey ? 1 : 0;
  }
  const int above = block_sum<THREADS>(n_above, sh.scratch, parity);
  const int ninf = block_sum<THREADS>(n_ninf, sh.scratch, parity);
  uint32_t T;
  int k_rem;
  if (above < k && above + ninf >= k) {
    T = kNegInfKey;
    k_rem = k - above;
  } else {
    const uint32_t floor_key = (above >= k) ? kNegInfKey + 1u : 0u;
    uint32_t mn = 0xFFFFFFFFu, mx = 0u;
    for (int i = threadIdx.x; i < n; i += THREADS) {
      const uint32_t kk = fkey(__ldg(v + i));
      mn = kk >= floor_key ? min(mn, kk) : mn;
      mx = kk >= floor_key ? max(mx, kk) : mx;
    }
    block_minmax<THREADS>(mn, mx, sh.mm, parity);
    int shift = (mn == mx) ? 0 : 32 - __clz(mn ^ mx);
    uint32_t prefix = (shift >= 32) ? 0u : (mx & ~((1u << shift) - 1u));
    k_rem = k;
    while (shift > 0) {
      const int d = min(kHistBits, shift);
      const int nbins = 1 << d;
      for (int i = threadIdx.x; i < nbins; i += THREADS) sh.hist[i] = 0;
      __syncthreads();
      const int ns = shift - d;
      for (int i = threadIdx.x; i < n; i += THREADS) {
        const uint32_t kk = fkey(__ldg(v + i));
        if (kk >= floor_key && prefix_match(kk, prefix, shift)) atomicAdd(&sh.hist[(kk >> ns) & (nbins - 1)], 1);
      }
      __syncthreads();
      pick_digit<THREADS>(sh, nbins, ns, prefix, k_rem, parity);
      prefix = sh.prefix;
      k_rem = sh.krem;
      shift = ns;
      __syncthreads();
    }
    T = prefix;
  }
  // Ordered compaction over per-thread contiguous chunks.
  const int chunk = (n + THREADS - 1) / THREADS;
  const int p0 = threadIdx.x * chunk;
  const int p1 = min(n, p0 + chunk);
  int gt = 0, eq = 0;
  for (int pos = p0; pos < p1; ++pos) {
    const uint32_t kk = fkey(__ldg(v + pos));
    gt += kk > T;
    eq += kk == T;
  }
  const int eq_before = block_excl_scan<THREADS>(eq, sh.scratch, parity);
  const int take_eq = max(0, min(eq, k_rem - eq_before));
  int o = block_excl_scan<THREADS>(gt + take_eq, sh.scratch, parity);
  const int32_t* cand_row = cand_idx ? cand_idx + row * cand_ld : nullptr;
  int32_t* oi = out_idx + row * k;
  float* ov = out_val + row * k;
  int e = eq_before;
  for (int pos = p0; pos < p1; ++pos) {
    const float x = __ldg(v + pos);
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
