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
// NaN: every NaN, of either sign, ranks above +inf and NaNs tie with one another (torch.topk's
// order: its radix keys send each NaN to the all-ones key). A NaN selected by the register kernel
// comes back as the canonical NaN (0x7FFFFFFF, the value of its key; rewriting it with its own bits
// costs registers the kernel does not have), elsewhere with its own bits. -0.0 ranks just below
// +0.0 (distinct keys, as in torch.topk on the GPU). So no key ranks below -inf, and the masked
// (-inf) tail of a row is the bottom of its order.
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
// topk_reg_kernel keeps a row of up to THREADS*ITEMS keys in registers (one read of the row),
// gathers the statistics of step 1 behind a single barrier, and as soon as the open histogram bin
// holds at most THREADS keys it ranks those keys directly instead of running further passes; the
// selected entries are staged in shared memory and written with 16-byte stores. For causal indexer
// rows the masked tail is known and is counted as -inf without being read.
// topk_gmem_kernel re-reads longer rows from global memory (L2) in each pass.
#pragma once
#include "common.cuh"

namespace dsv32 {
namespace topk {

constexpr uint32_t kNegInfKey = 0x007FFFFFu;  // key of -inf: below every finite value
constexpr uint32_t kNaNKey = 0xFFFFFFFFu;     // key of every NaN: above +inf (0xFF800000)
constexpr int kHistBits = 11;

// Order-preserving key: negative floats have all bits flipped, the others the sign bit raised. NaN is
// tested first: written as an OR with the sign mask, the non-NaN mapping may be compiled to a
// floating-point negate of the absolute value, which turns a NaN into the canonical NaN.
DSV32_DEV uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint32_t k = u ^ (static_cast<uint32_t>(static_cast<int32_t>(u) >> 31) | 0x80000000u);
  return f != f ? kNaNKey : k;
}

DSV32_DEV float fkey_inv(uint32_t k) {
  // top bit set: a positive float with its sign bit raised; clear: a negative float, all bits flipped
  const uint32_t flip = ~static_cast<uint32_t>(static_cast<int32_t>(k) >> 31) | 0x80000000u;
  return __uint_as_float(k ^ flip);
}

// Keys of a row fall into: "above" (> the -inf key: finite, +inf, NaN) and the -inf key. Masked
// -inf entries are counted, never histogrammed.
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
constexpr int kRegBits = 11;                // digit width of the register kernel's histograms
constexpr int kRegBins = 1 << kRegBits;
constexpr int kStageMax = 2048;             // outputs staged in shared memory (16-byte stores) up to this k

template <int THREADS>
struct RegShared {
  union {
    alignas(16) int hist[kRegBins];
    struct {
      int32_t idx[kStageMax];
      float val[kStageMax];
    } out;
  } u;
  uint32_t cand[32];       // keys of the last open histogram bin (at most 32)
  uint32_t red[4][32];     // per-warp partial statistics
  int scan[32];
  uint32_t prefix, T;
  int krem, bin_cnt, cand_n;
};

// Visible length of a row: positions >= valid are -inf without being read (causal rows of the
// indexer, whose masked tail is known). causal_m == 0: the whole row.
DSV32_DEV int row_valid(long long row, int n, int causal_m, long long causal_start) {
  if (causal_m <= 0) return n;
  const long long v = causal_start + (row % causal_m) + 1;
  return static_cast<int>(v < 0 ? 0 : (v > n ? n : v));
}

// Block-wide exclusive prefix sum (thread order) with a single barrier.
template <int THREADS>
DSV32_DEV int excl_scan_once(int v, int* buf) {
  constexpr int W = THREADS / 32;
  const int lane = threadIdx.x & 31;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) buf[threadIdx.x >> 5] = incl;
  __syncthreads();
  int before = 0;
  const int wid = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < W; ++i) before += (i < wid) ? buf[i] : 0;
  return before + incl - v;
}

// Copies k staged (index, value) pairs from shared memory to a row of the outputs, with 16-byte
// stores when the row is aligned for them.
template <int THREADS>
DSV32_DEV void copy_out_staged(const int32_t* sidx, const float* sval, int32_t* oi, float* ov, int k) {
  const int tid = threadIdx.x;
  if ((k & 3) == 0 && (reinterpret_cast<uintptr_t>(oi) & 15u) == 0 && (reinterpret_cast<uintptr_t>(ov) & 15u) == 0) {
    for (int j = tid; j < k / 4; j += THREADS) {
      reinterpret_cast<int4*>(oi)[j] = reinterpret_cast<const int4*>(sidx)[j];
      reinterpret_cast<float4*>(ov)[j] = reinterpret_cast<const float4*>(sval)[j];
    }
  } else {
    for (int j = tid; j < k; j += THREADS) {
      oi[j] = sidx[j];
      ov[j] = sval[j];
    }
  }
}

// A row given as the concatenation of n lists of len positions each (list j of row r at v[j] + r * ld,
// its candidate ids at id[j] + r * ld): the per-rank top-k lists of a key-sharded selection, read in
// place, possibly from other GPUs' memory. n == 0: rows are plain (vals / cand_idx addressing).
constexpr int kMaxParts = 16;
// ndst > 0: the selected row is written to each of ndst output pairs (out_idx[d], out_val[d], row-major
// [rows, k] like out_idx / out_val) instead of out_idx / out_val: a merged row block lands in every
// rank's output buffer (local or mapped from other GPUs) in one pass. Requires k <= kStageMax (the
// row is staged in shared memory and copied out once per destination).
struct RowParts {
  const float* v[kMaxParts];
  const int32_t* id[kMaxParts];
  int32_t* out_idx[kMaxParts];
  float* out_val[kMaxParts];
  long long ld;
  int len, n, ndst;
};

// Positions past n hold key 0 (below every real key): they never count as above -inf, never reach a
// histogram, and never equal a threshold, which is at least the -inf key.
// Causal rows: input row r is causal row r + causal_row0 (a batch of a larger problem).
// Segmented form: output row r' = blockIdx.x selects from segment r' % nseg (positions
// [seg0, seg0 + seg_len) of input row r' / nseg); nseg = 1, seg_len = n_total is the plain top-k.
// Each segment's list is written to out row r' (k entries); the nseg lists of an input row are
// contiguous, in segment order, so they form that row's candidate list for a merge pass.
// With parts.n > 0 the row is the concatenation of the parts (parts.len a multiple of ITEMS, so the
// ITEMS positions of a thread lie in one part) and candidate ids come from the parts.
// Six 256-thread or three 512-thread CTAs per SM (40 registers, some spilled to L1): the barriers
// between the selection phases are hidden by the other CTAs (4096 x 4096: 57.4 -> 53.1 us against
// four 256-thread CTAs; 2048 x 131072 staged: 1593 -> 1461 us against two 512-thread CTAs).
template <int THREADS, int ITEMS>
__global__ void __launch_bounds__(THREADS, THREADS == 256 ? 6 : 3) topk_reg_kernel(const float* __restrict__ vals, long long ld, int n_total,
                                                           const int32_t* __restrict__ cand_idx, long long cand_ld,
                                                           long long idx_offset, int k, int32_t* __restrict__ out_idx,
                                                           float* __restrict__ out_val, int causal_m,
                                                           long long causal_start, long long causal_row0,
                                                           int seg_len, int nseg,
                                                           const __grid_constant__ RowParts parts,
                                                           const int* __restrict__ row_len = nullptr) {
  constexpr int W = THREADS / 32;
  static_assert(ITEMS <= 32, "per-thread selection masks are 32-bit");
  __shared__ RegShared<THREADS> sh;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int wid = tid >> 5;
  // Causal rows are dealt out longest first (their visible length grows with the row), so the short
  // rows' copies fill the end of the launch instead of delaying the long selections.
  const long long out_row = (causal_m > 0 && nseg == 1) ? static_cast<long long>(gridDim.x) - 1 - blockIdx.x
                                                        : static_cast<long long>(blockIdx.x);
  const long long row = out_row / nseg;
  const int seg0 = static_cast<int>(out_row % nseg) * seg_len;
  const int n = min(seg_len, n_total - seg0);
  // row_len (candidate lists of the long-row filter, nseg = 1): row r holds row_len[r] >= k
  // candidates; a negative length marks a row finished elsewhere.
  int rl = n_total;
  if (row_len) {
    pdl_wait();
    rl = row_len[row];
    if (rl < 0) {
      pdl_launch_dependents();
      return;
    }
  }
  const int valid = max(0, min(min(n, rl), row_valid(row + causal_row0, n_total, causal_m, causal_start) - seg0));
  const int pos0 = tid * ITEMS;
  // This thread's ITEMS positions: their scores and (merge passes) candidate ids. The ids are only
  // needed at the end; the lambda recomputes their address there instead of holding it.
  auto thread_part = [&]() { return min((seg0 + min(pos0, max(n - 1, 0))) / max(parts.len, 1), parts.n - 1); };
  auto thread_ids = [&]() -> const int32_t* {
    if (parts.n > 0) {
      const int pj = thread_part();
      return parts.id[pj] + row * parts.ld + (seg0 + pos0 - pj * parts.len);
    }
    return cand_idx ? cand_idx + row * cand_ld + seg0 + pos0 : nullptr;
  };
  const float* tv;
  if (parts.n > 0) {
    const int pj = thread_part();
    tv = parts.v[pj] + row * parts.ld + (seg0 + pos0 - pj * parts.len);
  } else {
    tv = vals + row * ld + seg0 + pos0;
  }
  pdl_wait();
  pdl_launch_dependents();
  // 0. A row with at most k visible positions (a causal row that sees <= k keys) selects exactly its
  //    first k positions: no key ranks below the masked -inf tail, and the tail's ties go to the
  //    lowest positions. Output j is position j, copied straight to the outputs.
  if (valid <= k) {
    for (int d = 0; d < max(parts.ndst, 1); ++d) {
      int32_t* oi = (parts.ndst > 0 ? parts.out_idx[d] : out_idx) + out_row * k;
      float* ov = (parts.ndst > 0 ? parts.out_val[d] : out_val) + out_row * k;
      if (parts.n > 0) {
        for (int j = tid; j < k; j += THREADS) {
          const int pj = (seg0 + j) / parts.len;
          const long long off = row * parts.ld + (seg0 + j - pj * parts.len);
          oi[j] = parts.id[pj][off];
          ov[j] = j < valid ? __ldg(parts.v[pj] + off) : -INFINITY;
        }
      } else {
        const float* v = vals + row * ld + seg0;
        const int32_t* cand_row = cand_idx ? cand_idx + row * cand_ld + seg0 : nullptr;
        for (int j = tid; j < k; j += THREADS) {
          oi[j] = cand_row ? cand_row[j] : static_cast<int32_t>(j + seg0 + idx_offset);
          ov[j] = j < valid ? __ldg(v + j) : -INFINITY;
        }
      }
    }
    if (parts.ndst > 0) __threadfence_system();
    return;
  }
  for (int i = tid; i < kRegBins; i += THREADS) sh.u.hist[i] = 0;  // first radix pass
  uint32_t key[ITEMS];
  // Each thread owns ITEMS consecutive positions (position order = thread order). Positions in
  // [valid, n) are -inf without a read.
  if ((reinterpret_cast<uintptr_t>(tv) & 15u) == 0 && (ITEMS % 4) == 0 && pos0 + ITEMS <= valid) {
#pragma unroll
    for (int i = 0; i < ITEMS; i += 4) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(tv + i));
      key[i] = fkey(f.x);
      key[i + 1] = fkey(f.y);
      key[i + 2] = fkey(f.z);
      key[i + 3] = fkey(f.w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < ITEMS; ++i)
      key[i] = (pos0 + i < valid) ? fkey(__ldg(tv + i)) : (pos0 + i < n ? kNegInfKey : 0u);
  }
  // 1. Statistics of the keys above -inf behind one barrier (which also orders the histogram clear
  //    before pass 1), with the -inf and padding keys mapped to the top of the unsigned range for the
  //    minimum.
  {
    int na = 0;
    uint32_t mnw = 0xFFFFFFFFu, mx = 0u;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      na += key[i] > kNegInfKey ? 1 : 0;
      mnw = min(mnw, key[i] - (kNegInfKey + 1u));
      mx = max(mx, key[i]);
    }
    const uint32_t r0 = __reduce_add_sync(0xffffffffu, static_cast<uint32_t>(na));
    const uint32_t r2 = __reduce_min_sync(0xffffffffu, mnw);
    const uint32_t r3 = __reduce_max_sync(0xffffffffu, mx);
    if (lane == 0) {
      sh.red[0][wid] = r0;
      sh.red[2][wid] = r2;
      sh.red[3][wid] = r3;
    }
  }
  __syncthreads();
  // The threshold key T and krem, how many of the keys equal to T are taken (lowest positions first).
  // With fewer than k keys above -inf: all of them, then the lowest-position -inf entries (no key
  // ranks below -inf; padding keys 0 never reach T).
  uint32_t T = kNegInfKey;
  int krem;
  {
    int above = 0;
    uint32_t mnw = 0xFFFFFFFFu, mx = 0u;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      above += static_cast<int>(sh.red[0][w]);
      mnw = min(mnw, sh.red[2][w]);
      mx = max(mx, sh.red[3][w]);
    }
    krem = k - above;
    if (above >= k) {
      // 2. Radix select among the keys above -inf. Past the first pass the open bin is at most 2^21
      //    keys wide and never straddles the -inf key (a multiple of 2^23 plus 2^23 - 1), so a prefix
      //    match alone identifies the participants.
      const uint32_t mn = mnw + (kNegInfKey + 1u);
      int shift = (mn == mx) ? 0 : 32 - __clz(mn ^ mx);
      uint32_t prefix = (shift >= 32) ? 0u : (mx & ~((1u << shift) - 1u));
      krem = k;
      bool first = true, resolved = false;
      while (shift > 0) {
        const int d = min(kRegBits, shift);
        const int nbins = 1 << d;
        const int ns = shift - d;
        if (first) {
#pragma unroll
          for (int i = 0; i < ITEMS; ++i)
            if (key[i] > kNegInfKey) atomicAdd(&sh.u.hist[(key[i] >> ns) & (nbins - 1)], 1);
        } else {
          for (int i = tid; i < nbins; i += THREADS) sh.u.hist[i] = 0;
          __syncthreads();
          const uint32_t ph = prefix >> shift;
#pragma unroll
          for (int i = 0; i < ITEMS; ++i)
            if ((key[i] >> shift) == ph) atomicAdd(&sh.u.hist[(key[i] >> ns) & (nbins - 1)], 1);
        }
        first = false;
        __syncthreads();
        const int per = (nbins + THREADS - 1) / THREADS;
        int local = 0;
        if ((per & 3) == 0) {
          const int4* hv = reinterpret_cast<const int4*>(sh.u.hist + (nbins - (tid + 1) * per));
          for (int j = 0; j < per / 4; ++j) {
            const int4 h4 = hv[j];
            local += (h4.x + h4.y) + (h4.z + h4.w);
          }
        } else {
          for (int j = 0; j < per; ++j) {
            const int bin = nbins - 1 - (tid * per + j);
            if (bin >= 0) local += sh.u.hist[bin];
          }
        }
        const int before = excl_scan_once<THREADS>(local, sh.scan);
        if (before < krem && krem <= before + local) {
          int acc = before;
          for (int j = 0; j < per; ++j) {
            const int bin = nbins - 1 - (tid * per + j);
            const int c = sh.u.hist[bin];
            if (acc + c >= krem) {
              sh.prefix = prefix | (uint32_t(bin) << ns);
              sh.krem = krem - acc;
              sh.bin_cnt = c;
              sh.cand_n = 0;
              break;
            }
            acc += c;
          }
        }
        __syncthreads();
        prefix = sh.prefix;
        krem = sh.krem;
        const int cnt = sh.bin_cnt;
        shift = ns;
        if (shift > 0 && cnt <= 32) {
          const uint32_t ph = prefix >> shift;
#pragma unroll
          for (int i = 0; i < ITEMS; ++i)
            if ((key[i] >> shift) == ph) sh.cand[atomicAdd(&sh.cand_n, 1)] = key[i];
          __syncthreads();
          if (wid == 0) {
            const uint32_t mine = lane < cnt ? sh.cand[lane] : 0u;
            int g = 0, e = 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const uint32_t c = __shfl_sync(0xffffffffu, mine, j);
              g += (j < cnt && c > mine) ? 1 : 0;
              e += (j < cnt && c == mine) ? 1 : 0;
            }
            if (lane < cnt && g < krem && krem <= g + e) {
              sh.T = mine;
              sh.krem = krem - g;
            }
          }
          __syncthreads();
          T = sh.T;
          krem = sh.krem;
          resolved = true;
          break;
        }
      }
      if (!resolved) T = prefix;
    }
  }
  // 3. Ordered compaction: per-thread bit masks of the keys above / at the threshold, one scan of the
  //    packed counts gives every thread its output slot, and a popcount ranks each selected key.
  //    T is at least the -inf key, so padding keys are never selected.
  uint32_t gmask = 0, emask = 0;
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    gmask |= key[i] > T ? (1u << i) : 0u;
    emask |= key[i] == T ? (1u << i) : 0u;
  }
  const int eq = __popc(emask);
  const int packed = excl_scan_once<THREADS>((__popc(gmask) << 16) | eq, sh.scan);  // n <= 65535
  const int eq_before = packed & 0xFFFF;
  // keys equal to the threshold are taken in position order: this thread keeps its first `take`
  const int take = max(0, min(eq, krem - eq_before));
  while (__popc(emask) > take) emask &= ~(0x80000000u >> __clz(emask));  // drop the highest
  const uint32_t smask = gmask | emask;
  const int o = (packed >> 16) + min(eq_before, krem);
  int32_t* oi = out_idx + out_row * k;
  float* ov = out_val + out_row * k;
  const bool staged = k <= kStageMax;
  int32_t* si = staged ? sh.u.out.idx : oi;
  float* sv = staged ? sh.u.out.val : ov;
  // (one loop per id source: a per-entry choice in a single loop costs about 5% of the kernel)
  if (cand_idx || parts.n > 0) {
    const int32_t* ti = thread_ids();
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      if (smask & (1u << i)) {
        const int slot = o + __popc(smask & ((1u << i) - 1u));
        si[slot] = ti[i];
        sv[slot] = fkey_inv(key[i]);
      }
    }
  } else {
    const int32_t id0 = static_cast<int32_t>(pos0 + seg0 + idx_offset);  // ids are int32
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int slot = o + __popc(smask & ((1u << i) - 1u));
      if (smask & (1u << i)) {
        si[slot] = id0 + i;
        sv[slot] = fkey_inv(key[i]);
      }
    }
  }
  if (staged) {
    __syncthreads();
    if (parts.ndst > 0) {
      for (int d = 0; d < parts.ndst; ++d)
        copy_out_staged<THREADS>(sh.u.out.idx, sh.u.out.val, parts.out_idx[d] + out_row * k,
                                 parts.out_val[d] + out_row * k, k);
      __threadfence_system();  // the other GPUs' copies are complete before this CTA exits
    } else {
      copy_out_staged<THREADS>(sh.u.out.idx, sh.u.out.val, oi, ov, k);
    }
  }
}

// ---------------------------------------------------------------------------- long rows
// Positions at or past the row's visible length (causal rows) are -inf without being read. With
// row_state, only rows whose state is kRowFallback are selected (the others finished elsewhere).
constexpr int kRowFallback = -2;
template <int THREADS>
__global__ void __launch_bounds__(THREADS) topk_gmem_kernel(const float* __restrict__ vals, long long ld, int n,
                                                            const int32_t* __restrict__ cand_idx, long long cand_ld,
                                                            long long idx_offset, int k, int32_t* __restrict__ out_idx,
                                                            float* __restrict__ out_val, int causal_m,
                                                            long long causal_start, long long causal_row0,
                                                            const int* __restrict__ row_state) {
  __shared__ SelShared sh;
  int parity = 0;
  const long long row = blockIdx.x;
  const float* v = vals + row * ld;
  pdl_wait();
  pdl_launch_dependents();
  if (row_state && row_state[row] != kRowFallback) return;
  const int valid = row_valid(row + causal_row0, n, causal_m, causal_start);
  auto key_at = [&](int i) { return i < valid ? fkey(__ldg(v + i)) : kNegInfKey; };
  int n_above = 0;
  for (int i = threadIdx.x; i < n; i += THREADS) n_above += key_at(i) > kNegInfKey ? 1 : 0;
  const int above = block_sum<THREADS>(n_above, sh.scratch, parity);
  uint32_t T;
  int k_rem;
  if (above < k) {  // every key above -inf, then the lowest-position -inf entries (none ranks lower)
    T = kNegInfKey;
    k_rem = k - above;
  } else {
    const uint32_t floor_key = kNegInfKey + 1u;
    uint32_t mn = 0xFFFFFFFFu, mx = 0u;
    for (int i = threadIdx.x; i < n; i += THREADS) {
      const uint32_t kk = key_at(i);
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
        const uint32_t kk = key_at(i);
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
    const uint32_t kk = key_at(pos);
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
    const float x = pos < valid ? __ldg(v + pos) : -INFINITY;
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

// ---------------------------------------------------------------------------- long rows: filter
// Rows much longer than one register pass (the long-context indexer: 131072 keys) are reduced to a
// short candidate list in one read: a sample of the row gives a threshold T whose expected count of
// keys >= T is about 1.4 k; one pass over the row writes every key >= T, in position order, with its
// id, to the row's candidate list (at most `cap` = 2 k entries); the register kernel then selects the
// k largest of the list (row_len = its length). Every key >= the row's k-th largest is in the list
// whenever the list holds at least k keys, so the selection, ties included, equals the one over the
// whole row. A row whose list would hold fewer than k keys or more than cap (a sample far from the
// row's distribution, masked (-inf) keys among the k largest, at most k visible keys) is
// marked kRowFallback and selected by topk_gmem_kernel instead. One CTA per row.
constexpr int kFilterThreads = 512;
constexpr int kFilterItems = 16;
// Rows of at most this many keys use 256-thread CTAs (four per SM, a 4096-key sample): their fixed
// per-row work (sample, threshold search, barriers) weighs more, and more CTAs per SM hide it (random
// rows 4096 x 16384 301 -> 229 us, 4096 x 32768 -> 279 us, 2048 x 65536 235 -> 197 us). Longer rows keep
// 512 threads: with a 4096-key sample the threshold's error sends rows of 131072 to the fallback.
constexpr int kFilterShortN = 65536;

struct FilterShared {
  int hist[1 << kRegBits];
  int scan[32];
  uint32_t red[2][32];  // per-warp minimum / maximum key
  uint32_t cand[32];    // keys of the last open histogram bin (at most 32)
  uint32_t prefix, T;
  int krem, total, bin_cnt, cand_n;
};

// The c-th largest (1-based) key held by the block (ITEMS per thread; key 0 = no key), for
// 1 <= c <= number of keys. The bits common to the smallest and largest key are skipped (scores of
// one row share their sign and often their exponent), then 11-bit histogram passes over the keys
// matching the prefix found so far; as soon as the open bin holds at most 32 keys one warp ranks them.
template <int THREADS, int ITEMS>
DSV32_DEV uint32_t block_kth_key(const uint32_t (&key)[ITEMS], int c, FilterShared& sh) {
  constexpr int W = THREADS / 32;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  {
    uint32_t mn = 0xFFFFFFFFu, mx = 0u;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      if (key[i] != 0u) {
        mn = min(mn, key[i]);
        mx = max(mx, key[i]);
      }
    }
    mn = __reduce_min_sync(0xffffffffu, mn);
    mx = __reduce_max_sync(0xffffffffu, mx);
    if (lane == 0) {
      sh.red[0][wid] = mn;
      sh.red[1][wid] = mx;
    }
  }
  __syncthreads();
  uint32_t mn = 0xFFFFFFFFu, mx = 0u;
#pragma unroll
  for (int w = 0; w < W; ++w) {
    mn = min(mn, sh.red[0][w]);
    mx = max(mx, sh.red[1][w]);
  }
  int shift = (mn == mx) ? 0 : 32 - __clz(mn ^ mx);  // bits [shift, 32) common to every key
  uint32_t prefix = (shift >= 32) ? 0u : (mx & ~((1u << shift) - 1u));
  while (shift > 0) {
    const int d = min(kRegBits, shift);
    const int nbins = 1 << d;
    const int ns = shift - d;
    for (int i = threadIdx.x; i < nbins; i += THREADS) sh.hist[i] = 0;
    __syncthreads();  // (also orders the statistics' reads above and the previous pass's reads)
#pragma unroll
    for (int i = 0; i < ITEMS; ++i)
      if (key[i] != 0u && prefix_match(key[i], prefix, shift)) atomicAdd(&sh.hist[(key[i] >> ns) & (nbins - 1)], 1);
    __syncthreads();
    const int per = (nbins + THREADS - 1) / THREADS;  // consecutive bins per thread, descending
    int local = 0;
    for (int j = 0; j < per; ++j) {
      const int bin = nbins - 1 - (threadIdx.x * per + j);
      if (bin >= 0) local += sh.hist[bin];
    }
    const int before = excl_scan_once<THREADS>(local, sh.scan);
    if (before < c && c <= before + local) {
      int acc = before;
      for (int j = 0; j < per; ++j) {
        const int bin = nbins - 1 - (threadIdx.x * per + j);
        const int cnt = sh.hist[bin];
        if (acc + cnt >= c) {
          sh.prefix = prefix | (uint32_t(bin) << ns);
          sh.krem = c - acc;
          sh.bin_cnt = cnt;
          sh.cand_n = 0;
          break;
        }
        acc += cnt;
      }
    }
    __syncthreads();
    prefix = sh.prefix;
    c = sh.krem;
    shift = ns;
    const int cnt = sh.bin_cnt;
    if (shift > 0 && cnt <= 32) {
      // At most a warp's worth of keys share the digits found so far: one warp ranks them.
#pragma unroll
      for (int i = 0; i < ITEMS; ++i)
        if (key[i] != 0u && prefix_match(key[i], prefix, shift)) sh.cand[atomicAdd(&sh.cand_n, 1)] = key[i];
      __syncthreads();
      if (wid == 0) {
        const uint32_t mine = lane < cnt ? sh.cand[lane] : 0u;
        int g = 0, e = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const uint32_t o = __shfl_sync(0xffffffffu, mine, j);
          g += (j < cnt && o > mine) ? 1 : 0;
          e += (j < cnt && o == mine) ? 1 : 0;
        }
        if (lane < cnt && g < c && c <= g + e) sh.T = mine;  // every holder of this key writes it
      }
      __syncthreads();
      return sh.T;
    }
    __syncthreads();  // the next pass clears the histogram the scan above read
  }
  return prefix;
}

// The raw bits of ITEMS consecutive positions p .. p + ITEMS - 1 of a row; the bits of -inf past
// `valid` (masked positions, never selected by the filter).
constexpr uint32_t kNegInfBits = 0xFF800000u;
template <int ITEMS>
DSV32_DEV void load_bits(const float* v, int p, int valid, uint32_t (&bits)[ITEMS]) {
  if ((reinterpret_cast<uintptr_t>(v + p) & 15u) == 0 && p + ITEMS <= valid) {
#pragma unroll
    for (int i = 0; i < ITEMS; i += 4) {
      const uint4 f = __ldg(reinterpret_cast<const uint4*>(v + p + i));
      bits[i] = f.x;
      bits[i + 1] = f.y;
      bits[i + 2] = f.z;
      bits[i + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) bits[i] = (p + i < valid) ? __float_as_uint(__ldg(v + p + i)) : kNegInfBits;
  }
}

// Input row r of the batch: vals[r * ld .. + n) (positions past its causal visible length are -inf and
// never read; causal row index r + causal_row0), candidate ids cand_in[r * cand_in_ld + p] or
// p + idx_offset. Output: the row's list in cand_idx / cand_val[r * cap ..], its length in cand_n[r]
// (kRowFallback when the list does not apply).
template <int THREADS, int ITEMS>
__global__ void __launch_bounds__(THREADS, THREADS == 256 ? 4 : 2)
    topk_filter_kernel(const float* __restrict__ vals, long long ld, int n, const int32_t* __restrict__ cand_in,
                       long long cand_in_ld, long long idx_offset, int k, int causal_m, long long causal_start,
                       long long causal_row0, int32_t* __restrict__ cand_idx, float* __restrict__ cand_val,
                       int* __restrict__ cand_n, int cap) {
  constexpr int SPAN = THREADS * ITEMS;
  __shared__ FilterShared sh;
  const long long r = blockIdx.x;
  const int tid = threadIdx.x;
  const float* v = vals + r * ld;
  const int32_t* cin = cand_in ? cand_in + r * cand_in_ld : nullptr;
  const int valid = row_valid(r + causal_row0, n, causal_m, causal_start);
  pdl_wait();
  pdl_launch_dependents();
  if (valid <= k) {  // the k outputs include masked positions: the general selection handles them
    if (tid == 0) cand_n[r] = kRowFallback;
    return;
  }
  // 1. Sample: thread t reads ITEMS consecutive positions at t * stride (the whole visible row when it
  //    is at most SPAN long). The stride is rounded to a 16-byte multiple only when that keeps at least
  //    half of it, so short rows are sampled over their whole length.
  int stride = valid / THREADS;
  if (stride >= 2 * ITEMS) stride &= ~(ITEMS - 1);
  stride = max(stride, ITEMS);
  uint32_t key[ITEMS];
  load_bits<ITEMS>(v, tid * stride, valid, key);
  const int q0 = tid * stride;
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) key[i] = (q0 + i < valid) ? fkey(__uint_as_float(key[i])) : 0u;  // 0: no key
  // Sampled positions (s_n); every one holds a key (no real key is 0).
  int s_n = 0;
  {
    const int pos = max(0, min(ITEMS, valid - q0));
    const int cnt = __reduce_add_sync(0xffffffffu, pos);
    if ((tid & 31) == 0) sh.scan[tid >> 5] = cnt;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) s_n += sh.scan[w];
    __syncthreads();
  }
  // 2. Threshold: the c-th largest sampled key, c scaled so that about 1.4 k keys of the row reach it
  //    (exactly the k-th largest when the sample is the whole row). valid > k >= 1, so s_n >= 1.
  long long c_ll = (s_n >= valid) ? k : (7LL * k * s_n + 5LL * valid - 1) / (5LL * valid);
  if (c_ll < 1) c_ll = 1;
  if (c_ll > s_n) c_ll = s_n;
  const uint32_t T = block_kth_key<THREADS, ITEMS>(key, static_cast<int>(c_ll), sh);
  if (T <= kNegInfKey) {  // -inf among the candidates: the general selection
    if (tid == 0) cand_n[r] = kRowFallback;
    return;
  }
  // 3. Ordered compaction of every key >= T, SPAN positions per round, on the raw bits: key >= T is
  //    "not below T" as floats (NaN compares unordered, so it qualifies, as its key is the largest);
  //    otherwise the keys are formed. Positions past the visible length read as -inf, below T.
  int32_t* ci = cand_idx + r * cap;
  float* cv = cand_val + r * cap;
  // By value unless T is a NaN (NaNs of every payload qualify) or a signed zero (which the
  // floating-point compare does not tell apart).
  const bool by_value = T != kNaNKey && T != 0x80000000u && T != 0x7FFFFFFFu;
  const float tval = fkey_inv(T);
  int running = 0;
  uint32_t next[ITEMS];  // the following round's bits, requested before this round's scan
  load_bits<ITEMS>(v, tid * ITEMS, valid, next);
  for (int base = 0; base < valid; base += SPAN) {
    const int p = base + tid * ITEMS;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) key[i] = next[i];  // raw bits from here on
    if (base + SPAN < valid) load_bits<ITEMS>(v, p + SPAN, valid, next);
    uint32_t mask = 0;
    if (by_value) {  // x >= T or x unordered (NaN): one compare per value
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) mask |= !(__uint_as_float(key[i]) < tval) ? (1u << i) : 0u;
    } else {
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) mask |= fkey(__uint_as_float(key[i])) >= T ? (1u << i) : 0u;
    }
    const int cnt = __popc(mask);
    const int off = excl_scan_once<THREADS>(cnt, sh.scan);
    if (tid == THREADS - 1) sh.total = off + cnt;
    // This thread's candidates, lowest position first: one pass per candidate (a few % of the
    // positions), not a branch per position; the value is re-read (an L1 hit).
    int o = running + off;
    while (mask) {
      const int i = __ffs(mask) - 1;
      mask &= mask - 1;
      if (o < cap) {
        ci[o] = cin ? cin[p + i] : static_cast<int32_t>(p + i + idx_offset);
        cv[o] = __ldg(v + p + i);
      }
      ++o;
    }
    __syncthreads();
    running += sh.total;
    if (running > cap) break;  // (block-uniform) the list overflows: the row takes the fallback
  }
  if (tid == 0) cand_n[r] = (running >= k && running <= cap) ? running : kRowFallback;
}

}  // namespace topk
}  // namespace dsv32
