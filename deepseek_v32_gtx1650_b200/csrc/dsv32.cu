// C-ABI entry points of libdsv32_int8.so (declared in include/dsv32_int8.h).
//
// One translation unit: it includes every kernel header so all kernels share the single
// device error word g_dsv32_device_error. Host side: argument validation (the reference's
// asserts), TMA tensor-map encoding through the driver entry point (no -lcuda needed),
// per-device launch set-up, and the launches themselves.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <cudaTypedefs.h>

#include "../../include/dsv32_int8.h"
#include "act_quant.cuh"
#include "int8_gemm.cuh"
#include "int8_gemm_swap.cuh"
#include "int8_index.cuh"
#include "topk.cuh"
#include "producers.cuh"

namespace {

// act_quant lane split and loads in flight, by input width (fp32, 16-bit): values of a group per
// lane, and group slots per lane per iteration.
constexpr int kAqEplF32 = 8;
constexpr int kAqUnrollF32 = 2;
constexpr int kAqEpl16 = 8;
constexpr int kAqUnroll16 = 4;

thread_local std::string t_last_error;

int cuda_fail(cudaError_t e, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return DSV32_ERR_CUDA;
}

#define DSV32_CUDA_TRY(expr)                       \
  do {                                             \
    cudaError_t _e = (expr);                       \
    if (_e != cudaSuccess) return cuda_fail(_e, #expr); \
  } while (0)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct DeviceInfo {
  bool ready = false;
  bool sm100 = false;
  int num_sms = 0;
  int aq_blocks_per_sm[3] = {1, 1, 1};  // resident act_quant CTAs per SM, by input dtype
  uint8_t* noalloc_scratch = nullptr;   // device address of g_noalloc_scratch on this device
};

// Scratch of dsv32_int8_gemm_noalloc: the stream-K counters and partial-tile slots of small-M
// GEMMs, in a fixed array of the library's module instead of caller memory. Every GPU on which the
// library's module is loaded holds these 10 MiB until the process exits; all calls share them.
constexpr int64_t kNoAllocScratchBytes = int64_t(10) << 20;
constexpr int64_t kNoAllocTilesCap = 1024;  // counter capacity inside the static scratch
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
DeviceInfo g_dev[64];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

template <typename K>
cudaError_t set_smem(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// Per-device set-up: SM count, architecture check, dynamic smem opt-in for every kernel.
int device_setup(int* dev_out, DeviceInfo** info_out) {
  int dev = 0;
  DSV32_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return DSV32_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    int major = 0, minor = 0;
    DSV32_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    DSV32_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    DSV32_CUDA_TRY(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev));
    d.sm100 = (major == 10 && minor == 0);
    if (d.sm100) {
      using namespace dsv32;
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_kernel<256, false>, gemm::Smem<256>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_kernel<256, true>, gemm::Smem<256>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_kernel<128, false>, gemm::Smem<128>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_kernel<128, true>, gemm::Smem<128>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<16, false>, gemm::SwapSmem<16>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<16, true>, gemm::SwapSmem<16>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<32, false>, gemm::SwapSmem<32>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<32, true>, gemm::SwapSmem<32>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<64, false>, gemm::SwapSmem<64>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<64, true>, gemm::SwapSmem<64>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<16, false, 2>, gemm::SwapSmem<16, 2>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<16, true, 2>, gemm::SwapSmem<16, 2>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<32, false, 2>, gemm::SwapSmem<32, 2>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<32, true, 2>, gemm::SwapSmem<32, 2>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<64, false, 2>, gemm::SwapSmem<64, 2>::kAlloc));
      DSV32_CUDA_TRY(set_smem(gemm::int8_gemm_swap_kernel<64, true, 2>, gemm::SwapSmem<64, 2>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<64, 128, false>, index::Cfg<64, 128>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<64, 128, true>, index::Cfg<64, 128>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<32, 128, false>, index::Cfg<32, 128>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<32, 128, true>, index::Cfg<32, 128>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<16, 128, false>, index::Cfg<16, 128>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<16, 128, true>, index::Cfg<16, 128>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<64, 64, false>, index::Cfg<64, 64>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<64, 64, true>, index::Cfg<64, 64>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<32, 64, false>, index::Cfg<32, 64>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<32, 64, true>, index::Cfg<32, 64>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<16, 64, false>, index::Cfg<16, 64>::kAlloc));
      DSV32_CUDA_TRY(set_smem(index::int8_index_kernel<16, 64, true>, index::Cfg<16, 64>::kAlloc));
      {
        int nb = 0;
        DSV32_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &nb, act_quant_kernel<float, kAqEplF32, kAqUnrollF32>, 256, 0));
        d.aq_blocks_per_sm[DSV32_F32] = nb > 0 ? nb : 1;
        DSV32_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &nb, act_quant16_kernel<__nv_bfloat16, false, kAqUnroll16>, 256, 0));
        d.aq_blocks_per_sm[DSV32_BF16] = nb > 0 ? nb : 1;
        DSV32_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &nb, act_quant16_kernel<__half, false, kAqUnroll16>, 256, 0));
        d.aq_blocks_per_sm[DSV32_F16] = nb > 0 ? nb : 1;
      }
      if (!g_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        DSV32_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn) {
          t_last_error = "cuTensorMapEncodeTiled entry point not found";
          return DSV32_ERR_CUDA;
        }
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      }
    }
    d.ready = true;
  }
  if (!d.sm100) return DSV32_ERR_NO_DEVICE;
  *dev_out = dev;
  *info_out = &d;
  return DSV32_OK;
}

// Tiled int8 tensor map over a row-major array: dims listed innermost first, strides in bytes
// for dims 1.., box sizes per dim. Swizzle chosen from the inner box width (64 or 128 bytes).
int encode_i8_map(CUtensorMap* map, const void* ptr, int rank, const uint64_t* dims, const uint64_t* strides,
                  const uint32_t* box) {
  uint32_t estr[3] = {1, 1, 1};
  const CUtensorMapSwizzle swz = (box[0] == 128) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_error = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r));
    return DSV32_ERR_CUDA;
  }
  return DSV32_OK;
}

int launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return DSV32_OK;
}

// Launches a kernel with programmatic stream serialization (see pdl_wait in common.cuh): it may
// be scheduled while the previous kernel on the stream finishes, and waits for it before touching
// global memory. Arguments are converted to the kernel's parameter types.
template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t st, const char* what,
           Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return launch_check(what);
}

// launch() with the grid cut into clusters of `cluster` CTAs along x (grid a multiple of it).
template <typename... KArgs, typename... Args>
int launch_clusters(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t st,
                    const char* what, unsigned cluster, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return launch_check(what);
}

struct GemmPlan {
  int BN;
  int ew = dsv32::gemm::kEpiWarps;  // epilogue warps of the 128-row kernel (8; 16 measured slower)
  int swap_mn;  // > 0: decode-sized m on the swapped kernel, tokens padded to this many
  int pair = 1;  // 2: swapped kernel with a two-CTA cluster per tile, each CTA half of the K blocks
  int64_t tiles, units;
  int grid;
  bool split;
  int slot_rows;
  int64_t ws_tiles_cap;
  int64_t ws_bytes;  // workspace the stream-K schedule needs (0 when data-parallel)
};

// Tile width and schedule for an (m, n, k) problem on this device. m <= 64 runs the swapped kernel
// (weight rows on the UMMA M side, the tokens padded to 16, 32 or 64 on the N side) instead of
// padding the tokens to 128-row tiles. Stream-K only when there are fewer tiles than SMs
// (decode-sized m): there it is the only way to use every SM. With at least a wave of tiles, whole
// tiles per SM measured faster on B200 than splitting tiles (the partial-tile round trip through
// the workspace costs more than the tail wave it removes).
GemmPlan gemm_plan(int64_t m, int64_t n, int64_t k, int num_sms,
                   int64_t ws_tiles_cap = dsv32::gemm::kMaxSplitTiles, int slot_rows = dsv32::gemm::kBM) {
  GemmPlan p;
  p.swap_mn = m <= 16 ? 16 : m <= 32 ? 32 : m <= dsv32::gemm::kSwMaxM ? 64 : 0;
  // 128x256 tiles when they fill the GPU; otherwise 128x128 tiles (twice as many, so small-M problems
  // split K less: measured 25.1 -> 16.8 us at M=32 and 29.4 -> 20.6 us at M=512, N=7168, K=2048).
  // For full waves the wider tile wins (71 vs 106 us at 4096x2048x7168: a 128-wide MMA re-reads A
  // from shared memory twice as often).
  const int64_t tiles256 = ((m + 127) / 128) * (n / 256);
  p.BN = (n % 256 == 0 && tiles256 >= num_sms && !p.swap_mn) ? 256 : 128;
  p.tiles = ((m + 127) / 128) * ((n + p.BN - 1) / p.BN);  // swapped: n / 128 weight tiles, one token tile
  p.units = p.tiles * (k / 128);
  // The swapped kernel streams each tile's weights through one CTA unless the tiles cover under a
  // quarter of the SMs: whole tiles measured faster than spreading K blocks over every SM (m = 1, 8,
  // 32, 64 at n = 7168, k = 2048: 8.6 / 8.8 / 10.6 / 12.9 us against 12.3 / 12.4 / 13.9 / 16.5 us),
  // the partial-tile round trip through the workspace costing more than the SMs it brings in.
  p.split = (p.swap_mn ? p.tiles * 4 < num_sms : p.tiles < num_sms) && p.tiles <= ws_tiles_cap;
  p.slot_rows = slot_rows;
  p.ws_tiles_cap = ws_tiles_cap;
  if (p.split) {
    p.grid = static_cast<int>(p.units < num_sms ? p.units : num_sms);
    p.ws_bytes = p.swap_mn ? dsv32::gemm::swap_workspace_bytes(p.swap_mn, p.grid, ws_tiles_cap)
                           : dsv32::gemm::workspace_bytes(p.BN, p.grid, ws_tiles_cap, p.slot_rows);
  } else {
    p.grid = static_cast<int>(p.tiles < num_sms ? p.tiles : num_sms);
    p.ws_bytes = 0;
  }
  // Swapped kernel with whole tiles on at most half of the SMs: a CTA pair per tile, each streaming
  // half of the K blocks (one SM streams its tile's weights at ~50 GB/s, so the tile count sets the
  // bandwidth), the halves combined through the first CTA's shared memory (no workspace).
  if (p.swap_mn && !p.split && p.tiles * 2 <= num_sms && k / 128 >= 2) {
    p.pair = 2;
    p.grid = static_cast<int>(2 * p.tiles);
  }
  return p;
}

int gemm_check(const int8_t* a, const float* a_s, const int8_t* b, const float* b_s, const void* c, int c_dtype,
               int64_t m, int64_t n, int64_t k) {
  if (!a || !a_s || !b || !b_s || !c) return DSV32_ERR_INVALID_ARG;
  if (m < 1 || n < 1 || k < 1) return DSV32_ERR_INVALID_ARG;
  if (k % 128 != 0 || n % 128 != 0) return DSV32_ERR_UNSUPPORTED;
  if (c_dtype != DSV32_F32 && c_dtype != DSV32_BF16 && c_dtype != DSV32_F16) return DSV32_ERR_INVALID_ARG;
  if (m > (1LL << 31) - 1 || n > (1LL << 31) - 1 || k > (1LL << 31) - 1) return DSV32_ERR_UNSUPPORTED;
  if (!aligned16(a) || !aligned16(b) || !aligned16(c)) return DSV32_ERR_INVALID_ARG;
  return DSV32_OK;
}

// Encodes the operand tensor maps and launches the kernel for a plan (ws: NULL = data-parallel).
int gemm_launch(const GemmPlan& plan, const int8_t* a, const float* a_s, const int8_t* b, const float* b_s, void* c,
                int c_dtype, int64_t m, int64_t n, int64_t k, int32_t* partials, uint8_t* ws, void* stream) {
  CUtensorMap tmA, tmB;
  const uint64_t dimsA[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
  const uint64_t dimsB[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n)};
  const uint64_t strides[1] = {static_cast<uint64_t>(k)};
  const uint32_t boxA[2] = {128, static_cast<uint32_t>(plan.swap_mn ? plan.swap_mn : 128)};
  const uint32_t boxB[2] = {128, static_cast<uint32_t>(plan.BN)};
  if (int st = encode_i8_map(&tmA, a, 2, dimsA, strides, boxA)) return st;
  if (int st = encode_i8_map(&tmB, b, 2, dimsB, strides, boxB)) return st;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  using namespace dsv32::gemm;
  const int mi = static_cast<int>(m), ni = static_cast<int>(n), ki = static_cast<int>(k);
  const uint32_t ok = partials ? kOutF32 : static_cast<uint32_t>(c_dtype);
  const int cap = static_cast<int>(plan.ws_tiles_cap), sr = plan.slot_rows;
  const unsigned g = static_cast<unsigned>(plan.grid);
  if (plan.swap_mn) {
    const char* sw = "int8_gemm_swap_kernel launch";
    int32_t* const no_p = nullptr;
#define DSV32_SWAP_CASE(MN)                                                                                       \
  if (plan.swap_mn == MN && plan.pair == 1)                                                                       \
    return partials ? launch(int8_gemm_swap_kernel<MN, true>, g, kSwThreads, SwapSmem<MN>::kAlloc, st, sw, tmA, tmB, \
                             a_s, b_s, c, ok, mi, ni, ki, partials, ws, cap)                                      \
                    : launch(int8_gemm_swap_kernel<MN, false>, g, kSwThreads, SwapSmem<MN>::kAlloc, st, sw, tmA,   \
                             tmB, a_s, b_s, c, ok, mi, ni, ki, no_p, ws, cap);                                    \
  if (plan.swap_mn == MN && plan.pair == 2)                                                                       \
    return partials ? launch_clusters(int8_gemm_swap_kernel<MN, true, 2>, g, kSwThreads, SwapSmem<MN, 2>::kAlloc,  \
                                      st, sw, 2u, tmA, tmB, a_s, b_s, c, ok, mi, ni, ki, partials, ws, cap)       \
                    : launch_clusters(int8_gemm_swap_kernel<MN, false, 2>, g, kSwThreads, SwapSmem<MN, 2>::kAlloc, \
                                      st, sw, 2u, tmA, tmB, a_s, b_s, c, ok, mi, ni, ki, no_p, ws, cap);
    DSV32_SWAP_CASE(16)
    DSV32_SWAP_CASE(32)
    DSV32_SWAP_CASE(64)
#undef DSV32_SWAP_CASE
    return DSV32_ERR_UNSUPPORTED;
  }
  const char* what = "int8_gemm_kernel launch";
#define DSV32_GEMM_CASE(BNN, EWW)                                                                                  \
  if (plan.BN == BNN && plan.ew == EWW)                                                                            \
    return partials ? launch(int8_gemm_kernel<BNN, true, EWW>, g, threads_for(EWW), Smem<BNN>::kAlloc, st, what,    \
                             tmA, tmB, a_s, b_s, c, ok, mi, ni, ki, partials, ws, cap, sr)                         \
                    : launch(int8_gemm_kernel<BNN, false, EWW>, g, threads_for(EWW), Smem<BNN>::kAlloc, st, what,   \
                             tmA, tmB, a_s, b_s, c, ok, mi, ni, ki, static_cast<int32_t*>(nullptr), ws, cap, sr);
  DSV32_GEMM_CASE(256, 8)
  DSV32_GEMM_CASE(128, 8)
#undef DSV32_GEMM_CASE
  return DSV32_ERR_UNSUPPORTED;
}

int gemm_impl(const int8_t* a, const float* a_s, const int8_t* b, const float* b_s, void* c, int c_dtype, int64_t m,
              int64_t n, int64_t k, int32_t* partials, void* workspace, int64_t workspace_bytes, void* stream) {
  if (int st = gemm_check(a, a_s, b, b_s, c, c_dtype, m, n, k)) return st;
  if (workspace && !aligned16(workspace)) return DSV32_ERR_INVALID_ARG;
  int dev = 0;
  DeviceInfo* info = nullptr;
  if (int st = device_setup(&dev, &info)) return st;

  GemmPlan plan = gemm_plan(m, n, k, info->num_sms);
  if (plan.split && (!workspace || workspace_bytes < plan.ws_bytes)) {
    // No (large enough) workspace: data-parallel tiles.
    plan.split = false;
    plan.grid = static_cast<int>(plan.tiles < info->num_sms ? plan.tiles : info->num_sms);
  }
  uint8_t* ws = plan.split ? static_cast<uint8_t*>(workspace) : nullptr;

  return gemm_launch(plan, a, a_s, b, b_s, c, c_dtype, m, n, k, partials, ws, stream);
}

// Selection outputs the indexer writes itself: query rows m < m_triv (each sees at most k keys, so its
// top-k is its first k positions) get idx / val [row * k + j] = (j + key_offset, score or -inf).
struct IndexSel {
  int32_t* idx = nullptr;
  float* val = nullptr;
  int k = 0;
  int m_triv = 0;
  int key_offset = 0;
};

template <int H, int D>
int index_launch(const CUtensorMap& tmQ, const CUtensorMap& tmK, const float* w, const float* k_s, float* out,
                 int64_t batch, int64_t m, int64_t n, int causal, int64_t start, int64_t k_ld, int fill_masked,
                 const IndexSel& sel, int num_sms, cudaStream_t st) {
  using namespace dsv32::index;
  using C = Cfg<H, D>;
  const int64_t nqb = (m + C::QB - 1) / C::QB;
  const int64_t nt = (n + kKeysPerTile - 1) / kKeysPerTile;
  // Chunk the key tiles so that there are at least ~2 waves of work units.
  const int64_t want_units = 2LL * num_sms;
  int64_t chunks = (want_units + batch * nqb - 1) / (batch * nqb);
  if (chunks < 1) chunks = 1;
  if (chunks > nt) chunks = nt;
  int64_t tpc = (nt + chunks - 1) / chunks;
  chunks = (nt + tpc - 1) / tpc;
  const int64_t units = batch * nqb * chunks;
  if (units > 0x7FFFFFFFLL) return DSV32_ERR_UNSUPPORTED;
  const int64_t grid = units < num_sms ? units : num_sms;  // persistent: one CTA per SM
  auto* kernel = sel.m_triv > 0 ? int8_index_kernel<H, D, true> : int8_index_kernel<H, D, false>;
  return launch(kernel, static_cast<unsigned>(grid), kThreads, C::kAlloc, st,
                "int8_index_kernel launch", tmQ, tmK, w, k_s, out, static_cast<int>(m), static_cast<int>(n), causal,
                static_cast<long long>(start), static_cast<int>(tpc), static_cast<int>(chunks),
                static_cast<int>(units), static_cast<long long>(k_ld), fill_masked, sel.idx, sel.val, sel.k,
                sel.m_triv, sel.key_offset);
}

// k_ld: keys between the starts of consecutive batches of k and k_s (0: n, the contiguous layout).
// fill_masked == 0: key tiles no query of a block can see are left unwritten in `out`.
int index_impl(const int8_t* q, const float* w, const int8_t* k, const float* k_s, float* out, int64_t batch,
               int64_t m, int64_t n, int64_t heads, int64_t dim, int causal, int64_t start, int64_t k_ld,
               int fill_masked, void* stream, const IndexSel& sel = IndexSel{}) {
  if (!q || !w || !k || !k_s || !out) return DSV32_ERR_INVALID_ARG;
  if (batch < 1 || m < 1 || n < 1) return DSV32_ERR_INVALID_ARG;
  if (k_ld == 0) k_ld = n;
  if (k_ld < n) return DSV32_ERR_INVALID_ARG;
  if (!((heads == 16 || heads == 32 || heads == 64) && (dim == 64 || dim == 128))) return DSV32_ERR_UNSUPPORTED;
  // (keys stay below 2^30: the epilogue's per-query visibility bounds are kept within +-2^30)
  if (m * heads > (1LL << 31) - 1 || n >= (1LL << 30) || batch > 65535) return DSV32_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(w)) return DSV32_ERR_INVALID_ARG;
  int dev = 0;
  DeviceInfo* info = nullptr;
  if (int st = device_setup(&dev, &info)) return st;
  const int qb = static_cast<int>(256 / heads);
  CUtensorMap tmQ, tmK;
  const uint64_t dimsQ[3] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(m * heads),
                             static_cast<uint64_t>(batch)};
  const uint64_t strQ[2] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(m * heads * dim)};
  const uint32_t boxQ[3] = {static_cast<uint32_t>(dim), static_cast<uint32_t>(qb * heads), 1};
  const uint64_t dimsK[3] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(n), static_cast<uint64_t>(batch)};
  const uint64_t strK[2] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(k_ld * dim)};
  const uint32_t boxK[3] = {static_cast<uint32_t>(dim), 128, 1};
  if (int st = encode_i8_map(&tmQ, q, 3, dimsQ, strQ, boxQ)) return st;
  if (int st = encode_i8_map(&tmK, k, 3, dimsK, strK, boxK)) return st;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int S = info->num_sms;
#define DSV32_INDEX_CASE(HH, DD)                                                                              \
  if (heads == HH && dim == DD)                                                                               \
    return index_launch<HH, DD>(tmQ, tmK, w, k_s, out, batch, m, n, causal, start, k_ld, fill_masked, sel, S, st);
  DSV32_INDEX_CASE(64, 128)
  DSV32_INDEX_CASE(32, 128)
  DSV32_INDEX_CASE(16, 128)
  DSV32_INDEX_CASE(64, 64)
  DSV32_INDEX_CASE(32, 64)
  DSV32_INDEX_CASE(16, 64)
#undef DSV32_INDEX_CASE
  return DSV32_ERR_UNSUPPORTED;
}

// One launch of the register top-k: `rows` input rows, each split into nseg segments of seg_len
// (nseg = 1: whole rows of length n), k selections per segment into out [rows * nseg, k].
int topk_reg_launch(const float* vals, int64_t rows, int n, int64_t ld, const int32_t* cand_idx, int64_t cand_ld,
                    int64_t idx_offset, int k, int32_t* out_idx, float* out_val, int causal_m, int64_t causal_start,
                    int64_t causal_row0, int seg_len, int nseg, cudaStream_t st,
                    const dsv32::topk::RowParts& parts = dsv32::topk::RowParts{}, const int* row_len = nullptr) {
  using namespace dsv32::topk;
  const int64_t grid = rows * nseg;
  if (grid > 0x7FFFFFFFLL) return DSV32_ERR_UNSUPPORTED;
  const unsigned g = static_cast<unsigned>(grid);
  const long long cs = static_cast<long long>(causal_start), cr0 = static_cast<long long>(causal_row0);
  const char* what = "topk kernel launch";
  if (seg_len <= 256 * 4)
    return launch(topk_reg_kernel<256, 4>, g, 256, 0, st, what, vals, ld, n, cand_idx, cand_ld, idx_offset, k, out_idx,
                  out_val, causal_m, cs, cr0, seg_len, nseg, parts, row_len);
  if (seg_len <= 256 * 16)
    return launch(topk_reg_kernel<256, 16>, g, 256, 0, st, what, vals, ld, n, cand_idx, cand_ld, idx_offset, k,
                  out_idx, out_val, causal_m, cs, cr0, seg_len, nseg, parts, row_len);
  return launch(topk_reg_kernel<512, 16>, g, 512, 0, st, what, vals, ld, n, cand_idx, cand_ld, idx_offset, k, out_idx,
                out_val, causal_m, cs, cr0, seg_len, nseg, parts, row_len);
}

constexpr int kTopkRegMax = 512 * 16;                       // longest row a register pass holds
constexpr int64_t kTopkPreferredBytes = int64_t(256) << 20;  // workspace the library asks for, at most

// Long-row filter (topk_filter_kernel): plain rows longer than one register pass, k small enough
// that a list of 2 k candidates fits one register pass, and at least as many rows as SMs (with fewer
// rows the staged plan, which spreads each row's segments over several CTAs, is faster).
constexpr int kTopkFilterMinN = kTopkRegMax;
bool filter_shape(int64_t n, int64_t k) { return n > kTopkFilterMinN && 2 * k <= kTopkRegMax; }
constexpr int64_t kFilterEightN = 32768;  // rows up to this long: eight keys per thread (2048 sampled)
// List capacity 2 k: a list of at most 4096 candidates (k = 2048) is selected by the 256-thread
// register kernel, six CTAs per SM (3 k lists took the 512-thread one; with the 1.4 k target, random
// rows 4096 x 16384 368 -> 301 us, 2048 x 131072 364 -> 331 us).
int filter_cap(int k) { return (2 * k + 15) / 16 * 16; }
int64_t filter_per_row(int k) { return int64_t(filter_cap(k)) * 8 + 16; }

// Stage plan for rows longer than one register pass: each row is cut into equal segments of at most
// 8192 positions, every segment keeps its own top-k (a superset of the row's top-k within it), and the
// segment lists, contiguous and in position order, are merged by the next stage until one pass
// remains. Candidates keep global positions and their order, so ties resolve exactly as in a single
// pass. Stage outputs live in the caller's workspace: two ping-pong buffers of (id, value) candidates,
// `per_row` bytes per row of a row batch.
struct TopkPlan {
  int stages = 0;
  int nseg[8] = {}, seg[8] = {}, n[9] = {};
  bool ok = true;        // a staged plan exists (or none is needed)
  int64_t per_row = 0;   // workspace bytes per row (0: one register pass)
};

TopkPlan topk_plan(int n, int k, bool parts) {
  TopkPlan p;
  p.n[0] = n;
  while (p.n[p.stages] > kTopkRegMax) {
    const int cur = p.n[p.stages];
    const int nseg = (cur + kTopkRegMax - 1) / kTopkRegMax;
    // segment starts on 16-position boundaries when the first pass reads lists (a thread's 16
    // positions must not straddle two lists), else on 4-position (16-byte) boundaries
    const int align = (parts && p.stages == 0) ? 15 : 3;
    const int seg = ((cur + nseg - 1) / nseg + align) & ~align;
    if (p.stages == 8 || cur - (nseg - 1) * seg < k || static_cast<int64_t>(nseg) * k >= cur) {
      p.ok = false;
      return p;
    }
    p.nseg[p.stages] = nseg;
    p.seg[p.stages] = seg;
    p.n[p.stages + 1] = nseg * k;
    ++p.stages;
  }
  p.per_row = p.stages ? 2 * static_cast<int64_t>(p.n[1]) * 8 : 0;
  return p;
}

// Workspace bytes the top-k of `rows` rows of n positions wants (0: none), or -status.
int64_t topk_ws_bytes(int64_t rows, int64_t n, int64_t k, int nparts) {
  if (rows < 1 || n < 1 || k < 1 || k > n) return -DSV32_ERR_INVALID_ARG;
  if (n > (1LL << 31) - 1) return -DSV32_ERR_UNSUPPORTED;
  const TopkPlan p = topk_plan(static_cast<int>(n), static_cast<int>(k), nparts > 0);
  if (!p.ok && nparts > 0) return -DSV32_ERR_UNSUPPORTED;
  // plain rows: room for whichever of the staged plan and the filter the call takes (without either,
  // the long-row kernel needs nothing)
  int64_t per_row = p.ok ? p.per_row : 0;
  if (nparts == 0 && filter_shape(n, k)) per_row = std::max(per_row, filter_per_row(static_cast<int>(k)));
  if (per_row == 0) return 0;
  int64_t batch = kTopkPreferredBytes / per_row;
  if (batch < 1) batch = 1;
  if (batch > rows) batch = rows;
  return batch * per_row;
}

// causal_m > 0: row r (= b * causal_m + m) has its scores past key causal_start + m masked to -inf
// (the indexer's causal rows); those positions are treated as -inf without being read.
//
// Rows longer than one register pass run the staged plan in row batches sized to the workspace. With
// no workspace, or one smaller than a single row needs, or no staged plan (a segment shorter than k),
// plain rows go to the long-row kernel, which re-reads the row from L2 and needs no scratch; rows
// given as lists (parts) then return DSV32_ERR_UNSUPPORTED. Nothing is allocated here.
int topk_impl(const float* scores, int64_t rows, int64_t n, int64_t ld, const int32_t* cand_idx, int64_t cand_ld,
              int64_t idx_offset, int64_t k, int32_t* out_idx, float* out_val, void* workspace, int64_t ws_bytes,
              void* stream, int64_t causal_m = 0, int64_t causal_start = 0,
              const dsv32::topk::RowParts* parts = nullptr, const dsv32::topk::RowParts* dests = nullptr) {
  const dsv32::topk::RowParts no_parts{};
  const dsv32::topk::RowParts& p0 = parts ? *parts : no_parts;  // addressing of the first pass
  // dests (ndst > 0): the final pass writes each row to every destination pair instead of out_idx /
  // out_val (which then only has to be non-null); intermediate passes write the workspace as usual.
  // Destinations of row batch r0: the final addressing with out_idx / out_val of dests offset by r0 rows.
  auto final_parts = [&](const dsv32::topk::RowParts& base, int64_t r0) {
    dsv32::topk::RowParts f = base;
    if (dests) {
      f.ndst = dests->ndst;
      for (int d = 0; d < dests->ndst; ++d) {
        f.out_idx[d] = dests->out_idx[d] + r0 * k;
        f.out_val[d] = dests->out_val[d] + r0 * k;
      }
    }
    return f;
  };
  if ((!scores && !parts) || !out_idx || !out_val) return DSV32_ERR_INVALID_ARG;
  if (rows < 1 || n < 1 || k < 1 || k > n || (!parts && ld < n)) return DSV32_ERR_INVALID_ARG;
  if (cand_idx && cand_ld < n) return DSV32_ERR_INVALID_ARG;
  if (workspace && (!aligned16(workspace) || ws_bytes < 0)) return DSV32_ERR_INVALID_ARG;
  if (n > (1LL << 31) - 1 || rows > 0x7FFFFFFFLL) return DSV32_ERR_UNSUPPORTED;
  int dev = 0;
  DeviceInfo* info = nullptr;
  if (int st = device_setup(&dev, &info)) return st;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  using namespace dsv32::topk;
  const int nn = static_cast<int>(n), kk = static_cast<int>(k);
  const int cm = causal_m > 0 && causal_m <= 0x7FFFFFFFLL ? static_cast<int>(causal_m) : 0;
  if (n <= kTopkRegMax) {
    return topk_reg_launch(scores, rows, nn, ld, cand_idx, cand_ld, idx_offset, kk, out_idx, out_val, cm, causal_start,
                           0, nn, 1, st, final_parts(p0, 0));
  }
  if (!parts && workspace && filter_shape(n, k) && rows >= info->num_sms &&
      ws_bytes >= filter_per_row(kk)) {
    // Filter, per row batch: candidate lists (ids, values, lengths) in the workspace, the register
    // selection over each list, then the scratch-free kernel for the rows the lists do not cover.
    const int cap = filter_cap(kk);
    const int64_t fb = std::min<int64_t>(rows, ws_bytes / filter_per_row(kk));
    int32_t* ci = static_cast<int32_t*>(workspace);
    float* cv = reinterpret_cast<float*>(ci + fb * cap);
    int* cn = reinterpret_cast<int*>(cv + fb * cap);
    const long long cs = static_cast<long long>(causal_start);
    for (int64_t r0 = 0; r0 < rows; r0 += fb) {
      const int64_t rb = std::min<int64_t>(rows - r0, fb);
      const int32_t* cin = cand_idx ? cand_idx + r0 * cand_ld : nullptr;
      const bool short_rows = nn <= kFilterShortN;
      // Rows of at most 32768 keys (the local rows of a 4- or 8-GPU key split) sample 2048 keys with
      // eight per thread: random rows 4096 x 16384 228.8 -> 217.9 us, 4096 x 32768 278.2 -> 273.7 us;
      // longer rows keep sixteen per thread.
      if (int rc = nn <= kFilterEightN
                       ? launch(topk_filter_kernel<256, 8>, static_cast<unsigned>(rb), 256, 0, st,
                                "topk filter kernel launch", scores + r0 * ld, ld, nn, cin, cand_ld, idx_offset, kk, cm,
                                cs, static_cast<long long>(r0), ci, cv, cn, cap)
                   : short_rows ? launch(topk_filter_kernel<256, kFilterItems>, static_cast<unsigned>(rb), 256, 0, st,
                                       "topk filter kernel launch", scores + r0 * ld, ld, nn, cin, cand_ld, idx_offset,
                                       kk, cm, cs, static_cast<long long>(r0), ci, cv, cn, cap)
                              : launch(topk_filter_kernel<kFilterThreads, kFilterItems>, static_cast<unsigned>(rb),
                                       kFilterThreads, 0, st, "topk filter kernel launch", scores + r0 * ld, ld, nn,
                                       cin, cand_ld, idx_offset, kk, cm, cs, static_cast<long long>(r0), ci, cv, cn,
                                       cap))
        return rc;
      if (int rc = topk_reg_launch(cv, rb, cap, cap, ci, cap, 0, kk, out_idx + r0 * k, out_val + r0 * k, 0, 0, 0, cap,
                                   1, st, RowParts{}, cn))
        return rc;
      if (int rc = launch(topk_gmem_kernel<1024>, static_cast<unsigned>(rb), 1024, 0, st, "topk kernel launch",
                          scores + r0 * ld, ld, nn, cin, cand_ld, idx_offset, kk, out_idx + r0 * k, out_val + r0 * k,
                          cm, cs, static_cast<long long>(r0), static_cast<const int*>(cn)))
        return rc;
    }
    return DSV32_OK;
  }
  const TopkPlan plan = topk_plan(nn, kk, parts != nullptr);
  const int64_t batch = (plan.ok && workspace) ? std::min<int64_t>(rows, ws_bytes / plan.per_row) : 0;
  if (batch >= 1) {
    const int stages = plan.stages;
    const int64_t slot = batch * plan.n[1];  // candidates per buffer
    int32_t* bi[2] = {static_cast<int32_t*>(workspace), static_cast<int32_t*>(workspace) + slot};
    float* bv[2] = {reinterpret_cast<float*>(bi[1] + slot), reinterpret_cast<float*>(bi[1] + slot) + slot};
    for (int64_t r0 = 0; r0 < rows; r0 += batch) {
      const int64_t rb = (rows - r0 < batch) ? rows - r0 : batch;
      // stage 0 reads the caller's rows (causal tail skipped), later stages the candidate lists
      const float* in_v = scores ? scores + r0 * ld : nullptr;
      const int32_t* in_c = cand_idx ? cand_idx + r0 * cand_ld : nullptr;
      int64_t in_ld = ld, in_cld = cand_ld, off = idx_offset;
      int in_cm = cm;
      int64_t in_cs = causal_start;
      for (int sidx = 0; sidx < stages; ++sidx) {
        const int b = sidx & 1;
        dsv32::topk::RowParts pr = sidx == 0 ? p0 : no_parts;  // parts of this row batch
        for (int j = 0; j < pr.n; ++j) {
          pr.v[j] += r0 * pr.ld;
          pr.id[j] += r0 * pr.ld;
        }
        if (int rc = topk_reg_launch(in_v, rb, plan.n[sidx], in_ld, in_c, in_cld, off, kk, bi[b], bv[b], in_cm, in_cs,
                                     r0, plan.seg[sidx], plan.nseg[sidx], st, pr))
          return rc;
        in_v = bv[b];
        in_c = bi[b];
        in_ld = in_cld = plan.n[sidx + 1];
        off = 0;
        in_cm = 0;
        in_cs = 0;
      }
      if (int rc = topk_reg_launch(in_v, rb, plan.n[stages], in_ld, in_c, in_cld, off, kk, out_idx + r0 * k,
                                   out_val + r0 * k, in_cm, in_cs, r0, plan.n[stages], 1, st,
                                   final_parts(no_parts, r0)))
        return rc;
    }
    return DSV32_OK;
  }
  if (parts) {  // the long-row kernel reads plain rows only
    t_last_error = plan.ok ? "dsv32_topk_parts: rows longer than 8192 positions need a workspace of "
                                 "dsv32_topk_workspace_bytes() bytes"
                           : "dsv32_topk_parts: no staged plan for these list lengths";
    return DSV32_ERR_UNSUPPORTED;
  }
  return launch(topk_gmem_kernel<1024>, static_cast<unsigned>(rows), 1024, 0, st, "topk kernel launch", scores, ld, nn,
                cand_idx, cand_ld, idx_offset, kk, out_idx, out_val, cm, static_cast<long long>(causal_start), 0LL,
                static_cast<const int*>(nullptr));
}

}  // namespace

extern "C" {

int dsv32_abi_version(void) { return DSV32_ABI_VERSION; }

const char* dsv32_status_string(int status) {
  switch (status) {
    case DSV32_OK: return "ok";
    case DSV32_ERR_INVALID_ARG: return "invalid argument";
    case DSV32_ERR_UNSUPPORTED: return "unsupported shape";
    case DSV32_ERR_CUDA: return "CUDA error";
    case DSV32_ERR_DEVICE_TIMEOUT: return "kernel timed out on an internal wait";
    case DSV32_ERR_NO_DEVICE: return "current device is not an sm_100 GPU";
    default: return "unknown status";
  }
}

const char* dsv32_last_error_message(void) { return t_last_error.c_str(); }

int dsv32_act_quant(const void* x, int x_dtype, int64_t rows, int64_t n, int round_scale, int8_t* y, float* s,
                    void* stream) {
  if (!x || !y || !s) return DSV32_ERR_INVALID_ARG;
  if (rows < 0 || n < 0) return DSV32_ERR_INVALID_ARG;
  if (n % 128 != 0) return DSV32_ERR_UNSUPPORTED;
  if (x_dtype != DSV32_F32 && x_dtype != DSV32_BF16 && x_dtype != DSV32_F16) return DSV32_ERR_INVALID_ARG;
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(y) & 7u) != 0 || (reinterpret_cast<uintptr_t>(s) & 3u) != 0)
    return DSV32_ERR_INVALID_ARG;
  const int64_t groups = rows * (n / 128);
  if (groups == 0) return DSV32_OK;
  int dev = 0;
  DeviceInfo* info = nullptr;
  if (int st = device_setup(&dev, &info)) return st;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  using namespace dsv32;
  const int unroll = (x_dtype == DSV32_F32) ? kAqUnrollF32 : kAqUnroll16;
  const int threads = 256;
  const int gpw = 32 / (128 / ((x_dtype == DSV32_F32) ? kAqEplF32 : kAqEpl16));  // groups per warp slot
  const int64_t slots = (groups + gpw - 1) / gpw;
  const int64_t warps_needed = (slots + unroll - 1) / unroll;
  int64_t blocks = (warps_needed + (threads / 32) - 1) / (threads / 32);
  // One wave of resident CTAs, each looping over its share: no tail wave.
  const int64_t cap = static_cast<int64_t>(info->num_sms) * info->aq_blocks_per_sm[x_dtype];
  if (blocks > cap) blocks = cap;
  const unsigned g = static_cast<unsigned>(blocks);
  const char* what = "act_quant_kernel launch";
  if (x_dtype == DSV32_F32)
    return launch(act_quant_kernel<float, kAqEplF32, kAqUnrollF32>, g, threads, 0, st, what,
                  static_cast<const float*>(x), y, s, groups, round_scale);
  const char* what16 = "act_quant16_kernel launch";
  if (x_dtype == DSV32_BF16) {
    const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
    return round_scale ? launch(act_quant16_kernel<__nv_bfloat16, true, kAqUnroll16>, g, threads, 0, st, what16, xb,
                                y, s, groups)
                       : launch(act_quant16_kernel<__nv_bfloat16, false, kAqUnroll16>, g, threads, 0, st, what16,
                                xb, y, s, groups);
  }
  const __half* xh = static_cast<const __half*>(x);
  return round_scale ? launch(act_quant16_kernel<__half, true, kAqUnroll16>, g, threads, 0, st, what16, xh, y, s,
                              groups)
                     : launch(act_quant16_kernel<__half, false, kAqUnroll16>, g, threads, 0, st, what16, xh, y, s,
                              groups);
}

int dsv32_int8_gemm(const int8_t* a, const float* a_s, const int8_t* b, const float* b_s, void* c, int c_dtype,
                    int64_t m, int64_t n, int64_t k, void* workspace, int64_t workspace_bytes, void* stream) {
  return gemm_impl(a, a_s, b, b_s, c, c_dtype, m, n, k, nullptr, workspace, workspace_bytes, stream);
}

int64_t dsv32_int8_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m < 1 || n < 1 || k < 1 || k % 128 != 0 || n % 128 != 0) return -DSV32_ERR_UNSUPPORTED;
  int dev = 0;
  DeviceInfo* info = nullptr;
  if (int st = device_setup(&dev, &info)) return -st;
  return gemm_plan(m, n, k, info->num_sms).ws_bytes;
}

int dsv32_int8_gemm_noalloc(const int8_t* a, const float* a_s, const int8_t* b, const float* b_s, void* c,
                            int c_dtype, int64_t m, int64_t n, int64_t k, void* stream) {
  if (int st = gemm_check(a, a_s, b, b_s, c, c_dtype, m, n, k)) return st;
  int dev = 0;
  DeviceInfo* info = nullptr;
  if (int st = device_setup(&dev, &info)) return st;
  GemmPlan plan = gemm_plan(m, n, k, info->num_sms, kNoAllocTilesCap, dsv32::gemm::slot_rows_for(m));
  uint8_t* ws = nullptr;
  if (plan.split && plan.ws_bytes > kNoAllocScratchBytes) {
    // The balanced schedule would not fit the static scratch: whole tiles per SM instead, which
    // need no scratch (what dsv32_int8_gemm does without a workspace; same results up to fp32
    // summation order).
    plan.split = false;
    plan.grid = static_cast<int>(plan.tiles < info->num_sms ? plan.tiles : info->num_sms);
  }
  if (plan.split) {
    {
      // First call on this device (with it current): look up the array's device address once.
      std::lock_guard<std::mutex> lock(g_mu);
      if (!info->noalloc_scratch) {
        void* ptr = nullptr;
        DSV32_CUDA_TRY(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
        info->noalloc_scratch = static_cast<uint8_t*>(ptr);
      }
      ws = info->noalloc_scratch;
    }
    // The tile counters must start at zero; the slots need no clearing.
    DSV32_CUDA_TRY(cudaMemsetAsync(ws, 0, dsv32::gemm::counter_bytes(kNoAllocTilesCap),
                                   static_cast<cudaStream_t>(stream)));
  }
  return gemm_launch(plan, a, a_s, b, b_s, c, c_dtype, m, n, k, nullptr, ws, stream);
}

int dsv32_int8_gemm_partials(const int8_t* a, const float* a_s, const int8_t* b, const float* b_s, float* c,
                             int32_t* partials, int64_t m, int64_t n, int64_t k, void* workspace,
                             int64_t workspace_bytes, void* stream) {
  if (!partials) return DSV32_ERR_INVALID_ARG;
  return gemm_impl(a, a_s, b, b_s, c, DSV32_F32, m, n, k, partials, workspace, workspace_bytes, stream);
}

int dsv32_int8_index(const int8_t* q, const float* w, const int8_t* k, const float* k_s, float* out, int64_t batch,
                     int64_t m, int64_t n, int64_t heads, int64_t dim, int causal, int64_t start, int64_t k_ld,
                     void* stream) {
  return index_impl(q, w, k, k_s, out, batch, m, n, heads, dim, causal, start, k_ld, 1, stream);
}

int64_t dsv32_topk_workspace_bytes(int64_t rows, int64_t n, int64_t k, int nparts) {
  if (nparts < 0 || nparts > dsv32::topk::kMaxParts) return -DSV32_ERR_INVALID_ARG;
  return topk_ws_bytes(rows, n, k, nparts);
}

int dsv32_topk(const float* scores, int64_t rows, int64_t n, int64_t ld, const int32_t* cand_idx, int64_t cand_ld,
               int64_t idx_offset, int64_t k, int32_t* out_idx, float* out_val, void* workspace,
               int64_t workspace_bytes, void* stream) {
  return topk_impl(scores, rows, n, ld, cand_idx, cand_ld, idx_offset, k, out_idx, out_val, workspace,
                   workspace_bytes, stream);
}

int dsv32_device_alloc(int64_t bytes, void** ptr) {
  if (!ptr || bytes < 1) return DSV32_ERR_INVALID_ARG;
  *ptr = nullptr;
  const cudaError_t e = cudaMalloc(ptr, static_cast<size_t>(bytes));
  return e == cudaSuccess ? DSV32_OK : cuda_fail(e, "cudaMalloc");
}

int dsv32_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (!dst || !src || bytes < 0) return DSV32_ERR_INVALID_ARG;
  if (bytes == 0) return DSV32_OK;
  const cudaError_t e =
      cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? DSV32_OK : cuda_fail(e, "cudaMemcpyAsync");
}

int dsv32_device_free(void* ptr) {
  if (!ptr) return DSV32_OK;
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? DSV32_OK : cuda_fail(e, "cudaFree");
}

int dsv32_ipc_export(const void* ptr, void* handle) {
  if (!ptr || !handle) return DSV32_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == DSV32_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return DSV32_OK;
}

int dsv32_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return DSV32_ERR_INVALID_ARG;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? DSV32_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int dsv32_ipc_close(void* ptr) {
  if (!ptr) return DSV32_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? DSV32_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int dsv32_topk_parts(const float* const* part_vals, const int32_t* const* part_ids, int nparts, int64_t rows,
                     int64_t part_ld, int64_t part_len, int64_t k, int32_t* out_idx, float* out_val, void* workspace,
                     int64_t workspace_bytes, void* stream) {
  if (!part_vals || !part_ids || nparts < 1 || nparts > dsv32::topk::kMaxParts) return DSV32_ERR_INVALID_ARG;
  if (rows < 1 || part_len < 1 || part_ld < part_len || k < 1 || k > nparts * part_len) return DSV32_ERR_INVALID_ARG;
  if (part_len % 16 != 0 || nparts * part_len > (1LL << 30)) return DSV32_ERR_UNSUPPORTED;
  dsv32::topk::RowParts parts{};
  for (int j = 0; j < nparts; ++j) {
    if (!part_vals[j] || !part_ids[j]) return DSV32_ERR_INVALID_ARG;
    parts.v[j] = part_vals[j];
    parts.id[j] = part_ids[j];
  }
  parts.ld = part_ld;
  parts.len = static_cast<int>(part_len);
  parts.n = nparts;
  return topk_impl(nullptr, rows, nparts * part_len, part_ld, nullptr, 0, 0, k, out_idx, out_val, workspace,
                   workspace_bytes, stream, 0, 0, &parts);
}

int dsv32_topk_parts_to(const float* const* part_vals, const int32_t* const* part_ids, int nparts, int64_t rows,
                        int64_t part_ld, int64_t part_len, int64_t k, int32_t* const* out_idx, float* const* out_val,
                        int ndst, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!part_vals || !part_ids || nparts < 1 || nparts > dsv32::topk::kMaxParts) return DSV32_ERR_INVALID_ARG;
  if (!out_idx || !out_val || ndst < 1 || ndst > dsv32::topk::kMaxParts) return DSV32_ERR_INVALID_ARG;
  if (rows < 1 || part_len < 1 || part_ld < part_len || k < 1 || k > nparts * part_len) return DSV32_ERR_INVALID_ARG;
  if (part_len % 16 != 0 || nparts * part_len > (1LL << 30)) return DSV32_ERR_UNSUPPORTED;
  if (k > dsv32::topk::kStageMax) return DSV32_ERR_UNSUPPORTED;  // rows are staged once, copied per destination
  dsv32::topk::RowParts parts{}, dests{};
  for (int j = 0; j < nparts; ++j) {
    if (!part_vals[j] || !part_ids[j]) return DSV32_ERR_INVALID_ARG;
    parts.v[j] = part_vals[j];
    parts.id[j] = part_ids[j];
  }
  for (int d = 0; d < ndst; ++d) {
    if (!out_idx[d] || !out_val[d]) return DSV32_ERR_INVALID_ARG;
    dests.out_idx[d] = out_idx[d];
    dests.out_val[d] = out_val[d];
  }
  parts.ld = part_ld;
  parts.len = static_cast<int>(part_len);
  parts.n = nparts;
  dests.ndst = ndst;
  return topk_impl(nullptr, rows, nparts * part_len, part_ld, nullptr, 0, 0, k, out_idx[0], out_val[0], workspace,
                   workspace_bytes, stream, 0, 0, &parts, &dests);
}

int dsv32_int8_index_topk(const int8_t* q, const float* w, const int8_t* k, const float* k_s, float* scores,
                          int64_t batch, int64_t m, int64_t n, int64_t heads, int64_t dim, int causal, int64_t start,
                          int64_t k_ld, int scores_out, int64_t topk, int64_t key_offset, int32_t* out_idx,
                          float* out_val, void* workspace, int64_t workspace_bytes, void* stream) {
  if (topk < 1 || topk > n) return DSV32_ERR_INVALID_ARG;
  if (!out_idx || !out_val) return DSV32_ERR_INVALID_ARG;
  if (workspace && (!aligned16(workspace) || workspace_bytes < 0)) return DSV32_ERR_INVALID_ARG;
  // Without scores_out the masked tiles of causal rows stay unwritten: the selection never reads a
  // causal row past its visible length.
  // Causal single-batch calls: the leading rows that see at most topk keys (start + m + 1 <= topk) take
  // their first topk positions, which the indexer writes itself; the selection runs on the rest.
  IndexSel sel;
  if (causal && batch == 1 && m * topk <= 0x7FFFFFFFLL && key_offset >= 0 && key_offset + n <= 0x7FFFFFFFLL) {
    const int64_t mt = n <= topk ? m : std::min<int64_t>(m, std::max<int64_t>(0, topk - start));
    sel = IndexSel{out_idx, out_val, static_cast<int>(topk), static_cast<int>(mt), static_cast<int>(key_offset)};
  }
  if (int st = index_impl(q, w, k, k_s, scores, batch, m, n, heads, dim, causal, start, k_ld,
                          (scores_out || !causal) ? 1 : 0, stream, sel))
    return st;
  const int64_t mt = sel.m_triv;
  if (mt == m) return DSV32_OK;
  return topk_impl(scores + mt * n, batch * m - mt, n, n, nullptr, 0, key_offset, topk, out_idx + mt * topk,
                   out_val + mt * topk, workspace, workspace_bytes, stream, causal ? m - mt : 0, start + mt);
}

int dsv32_rotate_quant(const void* x, int x_dtype, int64_t rows, int rotate, int8_t* y, float* s,
                       const float* scale_mul, void* stream) {
  if (!x || !y || !s) return DSV32_ERR_INVALID_ARG;
  if (rows < 0) return DSV32_ERR_INVALID_ARG;
  if (x_dtype != DSV32_F32 && x_dtype != DSV32_BF16 && x_dtype != DSV32_F16) return DSV32_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(y) || (reinterpret_cast<uintptr_t>(s) & 3u) != 0) return DSV32_ERR_INVALID_ARG;
  if (rows == 0) return DSV32_OK;
  int dev = 0;
  DeviceInfo* info = nullptr;
  if (int st = device_setup(&dev, &info)) return st;
  using namespace dsv32;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // 4 vectors per warp slot, 8 warps per CTA; one resident wave of CTAs loops over the rest
  const int64_t want = (rows + 31) / 32;
  const int64_t cap = static_cast<int64_t>(info->num_sms) * 4;  // 4 resident CTAs per SM (64 registers)
  const unsigned g = static_cast<unsigned>(want < cap ? want : cap);
  const char* what = "rotate_quant_kernel launch";
  if (x_dtype == DSV32_F32)
    return launch(rotate_quant_kernel<float>, g, kRqThreads, 0, st, what, static_cast<const float*>(x), y, s, rows,
                  rotate, scale_mul);
  if (x_dtype == DSV32_BF16)
    return launch(rotate_quant_kernel<__nv_bfloat16>, g, kRqThreads, 0, st, what,
                  static_cast<const __nv_bfloat16*>(x), y, s, rows, rotate, scale_mul);
  return launch(rotate_quant_kernel<__half>, g, kRqThreads, 0, st, what, static_cast<const __half*>(x), y, s, rows,
                rotate, scale_mul);
}

int dsv32_weight_quant(const void* w, int w_dtype, int64_t n, int64_t k, int8_t* wq, float* ws, void* stream) {
  if (!w || !wq || !ws) return DSV32_ERR_INVALID_ARG;
  if (n < 0 || k < 0) return DSV32_ERR_INVALID_ARG;
  if (n % 128 != 0 || k % 128 != 0) return DSV32_ERR_UNSUPPORTED;
  if (w_dtype != DSV32_F32 && w_dtype != DSV32_BF16 && w_dtype != DSV32_F16) return DSV32_ERR_INVALID_ARG;
  if (!aligned16(w) || !aligned16(wq) || (reinterpret_cast<uintptr_t>(ws) & 3u) != 0) return DSV32_ERR_INVALID_ARG;
  const int64_t blocks = (n / 128) * (k / 128);
  if (blocks == 0) return DSV32_OK;
  if (blocks > 0x7FFFFFFFLL) return DSV32_ERR_UNSUPPORTED;
  int dev = 0;
  DeviceInfo* info = nullptr;
  if (int st = device_setup(&dev, &info)) return st;
  using namespace dsv32;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned g = static_cast<unsigned>(blocks);
  const char* what = "weight_quant_kernel launch";
  if (w_dtype == DSV32_F32)
    return launch(weight_quant_kernel<float>, g, kWqThreads, 0, st, what, static_cast<const float*>(w), wq, ws, n, k);
  if (w_dtype == DSV32_BF16)
    return launch(weight_quant_kernel<__nv_bfloat16>, g, kWqThreads, 0, st, what,
                  static_cast<const __nv_bfloat16*>(w), wq, ws, n, k);
  return launch(weight_quant_kernel<__half>, g, kWqThreads, 0, st, what, static_cast<const __half*>(w), wq, ws, n,
                k);
}

int dsv32_set_wait_limit(int64_t cycles) {
  const long long v = cycles > 0 ? static_cast<long long>(cycles) : DSV32_WAIT_LIMIT_CYCLES;
  DSV32_CUDA_TRY(cudaMemcpyToSymbol(g_dsv32_wait_limit, &v, sizeof(v)));
  return DSV32_OK;
}

int dsv32_device_status(int device, uint32_t* code) {
  if (!code) return DSV32_ERR_INVALID_ARG;
  int prev = 0;
  DSV32_CUDA_TRY(cudaGetDevice(&prev));
  if (prev != device) DSV32_CUDA_TRY(cudaSetDevice(device));
  cudaError_t e = cudaDeviceSynchronize();
  unsigned int v = 0;
  const unsigned int zero = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_dsv32_device_error, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_dsv32_device_error, &zero, sizeof(zero));
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "dsv32_device_status");
  *code = v;
  return v ? DSV32_ERR_DEVICE_TIMEOUT : DSV32_OK;
}

}  // extern "C"
