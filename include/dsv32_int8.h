/* dsv32_int8.h - C ABI of the B200 (sm_100a) INT8 hot-path kernels.
 *
 * This is the drop-in boundary for the three INT8 kernels of hamzak-27/deepseek-v32-gtx1650
 * (act_quant, int8_gemm, int8_index) plus the fused top-k selection the indexer feeds.
 * Every entry point takes plain device pointers, element counts and a CUDA stream
 * (passed as `void*`, a cudaStream_t; NULL = legacy default stream), launches
 * asynchronously on that stream and returns a status code. No torch types appear here.
 *
 * Conventions shared by all entry points
 *  - All pointers are device pointers to contiguous row-major arrays, 16-byte aligned.
 *  - Outputs and scratch are caller-allocated; inputs are never written. No compute entry point
 *    allocates device memory: kernels that need scratch (the stream-K GEMM, the staged top-k of long
 *    rows) take a caller workspace sized by a *_workspace_bytes() query. The only allocating calls
 *    are dsv32_device_alloc / dsv32_ipc_open, which exist to allocate and map memory.
 *  - Status codes: DSV32_OK on success; DSV32_ERR_* otherwise (see dsv32_status_string()).
 *    Argument errors are detected before any launch. Kernels that time out on an internal
 *    wait report it through dsv32_device_status().
 *  - Entry points may be called from any host thread; they keep no mutable global state
 *    apart from a per-device, mutex-guarded set-up cache.
 */
#ifndef DSV32_INT8_H_
#define DSV32_INT8_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSV32_ABI_VERSION 7

/* Status codes. */
#define DSV32_OK 0
#define DSV32_ERR_INVALID_ARG 1     /* null pointer, bad size, misaligned pointer */
#define DSV32_ERR_UNSUPPORTED 2     /* shape the reference asserts on (K % 128, N % 128, ...) */
#define DSV32_ERR_CUDA 3            /* a CUDA runtime/driver call failed */
#define DSV32_ERR_DEVICE_TIMEOUT 4  /* a kernel gave up on an internal wait (dsv32_device_status) */
#define DSV32_ERR_NO_DEVICE 5       /* current device is not an sm_100 GPU */

/* Element types. */
#define DSV32_F32 0
#define DSV32_BF16 1
#define DSV32_F16 2

/* act_quant: replaces kernels.py:55 act_quant(x, round_scale, block_m) and its kernel
 * kernels.py:37-52 (oracle reference.py:8-15).
 * x [rows, n] (x_dtype: DSV32_F32 / DSV32_BF16 / DSV32_F16), n % 128 == 0.
 * y [rows, n] int8; s [rows, n / 128] fp32. Per 128-wide group: s = max(amax, 1e-4) * (1/127),
 * or its ue8m0 power of two when round_scale != 0; y = clamp(round_half_even(x / s), +-127). */
int dsv32_act_quant(const void* x, int x_dtype, int64_t rows, int64_t n, int round_scale, int8_t* y, float* s,
                    void* stream);

/* int8_gemm: replaces kernels.py:109 int8_gemm(a, a_s, b, b_s, out_dtype, version) and its kernel
 * kernels.py:71-101 (oracle reference.py:18-24).
 * a [m, k] int8, a_s [m, k/128] fp32, b [n, k] int8, b_s [n/128, k/128] fp32,
 * c [m, n] of c_dtype (DSV32_F32 / DSV32_BF16 / DSV32_F16). k % 128 == 0, n % 128 == 0, any m >= 1.
 * c[i, j] = sum_kb fp32(A_kb . B_kb) * (a_s[i, kb] * b_s[j / 128, kb]), accumulated in fp32.
 * workspace: device scratch of at least dsv32_int8_gemm_workspace_bytes(m, n, k) bytes, zero-filled
 * before its first use; every completed launch leaves it reusable for any shape (after a launch that
 * reported DSV32_ERR_DEVICE_TIMEOUT, zero it again). It lets the kernel balance K-blocks over all SMs
 * (stream-K). NULL or too small: the kernel runs whole tiles per SM instead (same results up to fp32
 * summation order). One workspace must not serve two launches that may run concurrently. */
int dsv32_int8_gemm(const int8_t* a, const float* a_s, const int8_t* b, const float* b_s, void* c, int c_dtype,
                    int64_t m, int64_t n, int64_t k, void* workspace, int64_t workspace_bytes, void* stream);

/* Bytes of workspace dsv32_int8_gemm uses for (m, n, k) on the current device (0: none needed);
 * a negative value is -status on error. */
int64_t dsv32_int8_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k);

/* Debug form of dsv32_int8_gemm (same tensor-core path and schedule): also writes the exact int32
 * partial of every 128-wide K block, partials [k/128, m, n] int32, and c [m, n] fp32. For parity
 * tests. */
int dsv32_int8_gemm_partials(const int8_t* a, const float* a_s, const int8_t* b, const float* b_s, float* c,
                             int32_t* partials, int64_t m, int64_t n, int64_t k, void* workspace,
                             int64_t workspace_bytes, void* stream);

/* int8_gemm for callers that cannot allocate device memory. No counterpart in the reference.
 * Some hosts own every byte of device memory (an inference engine that plans all buffers into its
 * own arena and forbids plugins from calling cudaMalloc, or a process running under a fixed memory
 * budget), so they cannot hand dsv32_int8_gemm a workspace. This variant takes the same inputs and
 * output and allocates nothing: its scratch is a 10 MiB array inside the library, present on every
 * GPU that loads the library until the process exits. It computes what dsv32_int8_gemm computes.
 *  - The first call on a device (with that device current) looks up the array's address.
 *  - Each call clears the array's tile counters on `stream` before the kernel.
 *  - All calls share the one array: calls that may overlap on the GPU (other streams, other host
 *    threads) race and must be serialised by the caller.
 *  - Problems with at least one wave of 128-row tiles (one per SM) need no scratch and run at any
 *    size. Smaller problems spread their K blocks over all SMs through the scratch; those whose
 *    spread would need more than 10 MiB (for example m = 128 with n = 7168) run whole tiles per SM
 *    instead, which needs no scratch (same results up to fp32 summation order, as dsv32_int8_gemm
 *    without a workspace). */
int dsv32_int8_gemm_noalloc(const int8_t* a, const float* a_s, const int8_t* b, const float* b_s, void* c,
                            int c_dtype, int64_t m, int64_t n, int64_t k, void* stream);

/* int8_index: replaces kernels.py:165 int8_index(q, w, k, k_s, causal, start, ...) and its kernel
 * kernels.py:134-162 (oracle reference.py:27-34).
 * q [batch, m, heads, dim] int8, w [batch, m, heads] fp32, k [batch, n, dim] int8, k_s [batch, n] fp32,
 * out [batch, m, n] fp32. (heads, dim) in {16, 32, 64} x {64, 128}.
 * out[b, i, j] = k_s[b, j] * sum_h w[b, i, h] * relu(q[b, i, h, :] . k[b, j, :]);
 * causal != 0: out = -inf where j > start + i (start may be negative: a key shard whose first
 * key lies past some queries' positions).
 * k_ld: keys between the first keys of consecutive batches, for k (k_ld * dim bytes) and k_s (k_ld
 * floats); 0 means n (contiguous). A key cache [batch, capacity, dim] holding n <= capacity valid
 * keys is read in place with k_ld = capacity. */
int dsv32_int8_index(const int8_t* q, const float* w, const int8_t* k, const float* k_s, float* out, int64_t batch,
                     int64_t m, int64_t n, int64_t heads, int64_t dim, int causal, int64_t start, int64_t k_ld,
                     void* stream);

/* Bytes of workspace the top-k selection of `rows` rows of n positions uses on the current device
 * (0: none). nparts = 0 for dsv32_topk / dsv32_int8_index_topk rows, else the list count of a
 * dsv32_topk_parts call (n = nparts * part_len). Rows of at most 8192 positions need none. Longer
 * rows are selected in stages through the workspace, in row batches sized to whatever is passed
 * (the returned size covers up to 256 MB of rows; less works down to one row's share). A negative
 * value is -status: -DSV32_ERR_UNSUPPORTED when rows given as lists cannot be selected at all. */
int64_t dsv32_topk_workspace_bytes(int64_t rows, int64_t n, int64_t k, int nparts);

/* Top-k selection per row: replaces torch.topk(scores, k) on the indexer output
 * (test_kernels.py:125, bench_indexer_e2e.py:72-77).
 * Row r of the input is scores[r * ld + 0 .. n). Selects the k largest values (ties at the k-th
 * value: lowest position first) and writes them in increasing position order. Order as torch.topk
 * on the GPU: every NaN (either sign) above +inf, NaNs equal to one another; -0.0 below +0.0. A
 * selected NaN is written as a NaN (possibly the canonical 0x7FFFFFFF); other values bit for bit:
 * out_idx [rows, k] int32, out_val [rows, k] fp32. The index written for position p is
 * cand_idx[r * cand_ld + p] when cand_idx is non-NULL (merging candidate lists), else p + idx_offset
 * (a shard's first global key). Requires 1 <= k <= n.
 * workspace: 16-byte aligned device scratch of workspace_bytes (dsv32_topk_workspace_bytes); its
 * contents need no initialisation. NULL or smaller than one row's share: rows longer than 8192 are
 * selected by a kernel that re-reads them from L2 instead (slower, no scratch). One workspace must
 * not serve two launches that may run concurrently. */
int dsv32_topk(const float* scores, int64_t rows, int64_t n, int64_t ld, const int32_t* cand_idx, int64_t cand_ld,
               int64_t idx_offset, int64_t k, int32_t* out_idx, float* out_val, void* workspace,
               int64_t workspace_bytes, void* stream);

/* Indexer + top-k in one call (bench_indexer_e2e.py:54-57,72-77): scores are written to the
 * caller's `scores` buffer [batch, m, n] fp32, then the top `topk` keys of every (batch, query) row
 * are selected as dsv32_topk does, with index = key position + key_offset (a key shard's first
 * global key; 0 for a whole cache). k_ld as in dsv32_int8_index.
 * scores_out != 0: `scores` holds the full scores on return (-inf where masked). scores_out == 0:
 * `scores` is scratch, and with causal != 0 its masked entries are left unwritten (the selection
 * never reads a causal row past its visible length). With causal != 0 and batch == 1, the rows
 * that see at most topk keys (query m with start + m < topk) select their first topk positions;
 * the indexer writes those rows' outputs itself (and their scores only when scores_out != 0).
 * workspace / workspace_bytes: the selection's scratch, as for dsv32_topk (rows = batch * m).
 * out_idx / out_val [batch, m, topk]. Requires 1 <= topk <= n. */
int dsv32_int8_index_topk(const int8_t* q, const float* w, const int8_t* k, const float* k_s, float* scores,
                          int64_t batch, int64_t m, int64_t n, int64_t heads, int64_t dim, int causal, int64_t start,
                          int64_t k_ld, int scores_out, int64_t topk, int64_t key_offset, int32_t* out_idx,
                          float* out_val, void* workspace, int64_t workspace_bytes, void* stream);

/* Synchronises `device`, then reads and clears its kernel error word. *code = 0 if no kernel
 * gave up on an internal wait since the last call; else (kernel_id << 16) | site. Returns
 * DSV32_ERR_DEVICE_TIMEOUT when *code != 0. */
int dsv32_device_status(int device, uint32_t* code);

/* Bound, in SM clock cycles, after which a kernel gives up on an internal pipeline wait (a TMA load
 * or MMA that never completes), records (kernel_id << 16) | site for dsv32_device_status(), lets its
 * issued copies and MMAs land and returns; for the current device, for launches that follow.
 * cycles <= 0 restores the default (2e9, about a second). Failure-detection tests set a few hundred
 * cycles so that ordinary waits run out; the context stays usable. Not for use while kernels of the
 * library run on the device. */
int dsv32_set_wait_limit(int64_t cycles);

/* Human-readable text for a status code (static storage). */
const char* dsv32_status_string(int status);

/* Text of the last CUDA error seen by an entry point on this host thread (static per thread). */
const char* dsv32_last_error_message(void);

/* Indexer operand producer: replaces hadamard_quant.py:84-103 rotate_quant_kmajor / fwht_quant_kmajor
 * (row-major output; the K-major packing of kernels_v2 is a host-side view). x [rows, 128] of
 * x_dtype (DSV32_F32 / DSV32_BF16 / DSV32_F16), 16-byte aligned. rotate != 0: each vector is
 * multiplied by the 128-point Hadamard matrix scaled by 128^-1/2 (butterfly form, fp32), then
 * quantised per vector: s[r] = max(amax, 1e-4) * fl32(1/127), y[r, :] = clamp(rint(x / s), -127, 127)
 * (hadamard_quant.py:63-81). rotate == 0: the quantisation alone. y int8 [rows, 128], s fp32 [rows].
 * scale_mul: NULL, or fp32 [rows]; then s[r] = scale_mul[r] * scale of vector r, one fp32 rounding
 * (the indexer's head weights take the query scales this way, bench_indexer_e2e.py:55). */
int dsv32_rotate_quant(const void* x, int x_dtype, int64_t rows, int rotate, int8_t* y, float* s,
                       const float* scale_mul, void* stream);

/* Weight block quantiser for the GEMM's B operand (test_kernels.py:80-82, bench.py:43-44; the
 * reference computes it inline in torch): w [n, k] of w_dtype, n % 128 == 0, k % 128 == 0, 16-byte
 * aligned. Per 128 x 128 block: ws = max(amax, 1e-4) / 127 (fp32 division), wq = clamp(rint(w / ws),
 * -127, 127). wq int8 [n, k], ws fp32 [n/128, k/128]. */
int dsv32_weight_quant(const void* w, int w_dtype, int64_t n, int64_t k, int8_t* wq, float* ws, void* stream);

/* Merge of key-sharded selections (the exchange step of a key-range sharded indexer; the reference
 * runs on one GPU and has no such step, its single-GPU selection is test_kernels.py:125): row r is
 * the concatenation of nparts lists, list j at part_vals[j] + r * part_ld (part_len scores) with
 * their global key ids at part_ids[j] + r * part_ld. Selects as dsv32_topk does (ties: lower
 * position in the concatenation first) and writes the ids from the lists. The lists are read in
 * place and may live in other GPUs' memory (dsv32_ipc_open). 1 <= nparts <= 16, part_len % 16 == 0,
 * 1 <= k <= nparts * part_len. out_idx / out_val [rows, k]. Rows longer than 8192 positions need
 * the workspace dsv32_topk_workspace_bytes(rows, nparts * part_len, k, nparts) reports (at least one
 * row's share); without it they return DSV32_ERR_UNSUPPORTED before any launch. */
int dsv32_topk_parts(const float* const* part_vals, const int32_t* const* part_ids, int nparts, int64_t rows,
                     int64_t part_ld, int64_t part_len, int64_t k, int32_t* out_idx, float* out_val, void* workspace,
                     int64_t workspace_bytes, void* stream);

/* dsv32_topk_parts writing each selected row to ndst output pairs (out_idx[d], out_val[d], each
 * [rows, k]) instead of one: a rank's merged row block goes straight into every rank's output buffer
 * (local, or mapped from another GPU with dsv32_ipc_open) in one pass, in place of all-gathering the
 * merged blocks (same role as dsv32_topk_parts; no reference counterpart). 1 <= ndst <= 16,
 * k <= 2048. The writes to other GPUs are complete when the kernel is; the caller orders them
 * before any rank reads its output (a collective after the call). */
int dsv32_topk_parts_to(const float* const* part_vals, const int32_t* const* part_ids, int nparts, int64_t rows,
                        int64_t part_ld, int64_t part_len, int64_t k, int32_t* const* out_idx, float* const* out_val,
                        int ndst, void* workspace, int64_t workspace_bytes, void* stream);

/* Device memory another process on the node can map: cudaMalloc on the current device (the pointer
 * is the base of its allocation, as IPC export requires), and its release. */
int dsv32_device_alloc(int64_t bytes, void** ptr);
int dsv32_device_free(void* ptr);

/* One asynchronous copy of `bytes` bytes on `stream` (cudaMemcpyAsync, any direction; between GPUs
 * the copy engines move it over NVLink): the merge of key-sharded lists pulls the other ranks' rows
 * into this GPU's memory with it (no reference counterpart). */
int dsv32_copy_async(void* dst, const void* src, int64_t bytes, void* stream);

/* CUDA IPC of such an allocation: export writes its DSV32_IPC_HANDLE_BYTES-byte handle; open maps a
 * handle exported by another process (peer access enabled on first use), close unmaps it. */
#define DSV32_IPC_HANDLE_BYTES 64
int dsv32_ipc_export(const void* ptr, void* handle);
int dsv32_ipc_open(const void* handle, void** ptr);
int dsv32_ipc_close(void* ptr);

/* DSV32_ABI_VERSION of the loaded library. */
int dsv32_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* DSV32_INT8_H_ */
