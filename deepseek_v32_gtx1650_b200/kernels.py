"""Drop-in replacements for the reference's kernels.py API, backed by libdsv32_int8.so (sm_100a).

Same names, argument meaning, return shapes and assert behaviour as the reference
(kernels.py:55 act_quant, :109 int8_gemm, :165 int8_index). Tuning keywords of the Triton
versions (block_m, version, block_q, block_n, num_warps) are accepted and ignored: tile
shapes are fixed per shape class inside the CUDA library.

Every op runs the CUDA library on the input's device and current stream; there is no CPU
path. Calling with CPU tensors raises, as the reference's Triton launch would.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

GROUP = 128  # quantisation block (kernels.py:19)

_DT = {torch.float32: _lib.DSV32_F32, torch.bfloat16: _lib.DSV32_BF16, torch.float16: _lib.DSV32_F16}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


class _OnDevice:
    """Make t's device current for the library call (a no-op when it already is)."""
    __slots__ = ("idx", "prev")

    def __init__(self, t: torch.Tensor):
        self.idx = t.device.index

    def __enter__(self):
        self.prev = torch.cuda.current_device()
        if self.prev != self.idx:
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev != self.idx:
            torch.cuda.set_device(self.prev)


# GEMM workspace per (device, stream): zero-filled once, left reusable by every launch. Keyed by
# stream because two launches sharing one workspace must not overlap on the GPU.
_GEMM_WS: dict = {}


def _gemm_workspace(dev: torch.device, stream: int, M: int, N: int, K: int):
    nbytes = int(_lib.load().dsv32_int8_gemm_workspace_bytes(M, N, K))
    if nbytes <= 0:
        return None, 0
    key = (dev.index, stream)
    ws = _GEMM_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _GEMM_WS[key] = ws
    return ws.data_ptr(), ws.numel()


# Top-k workspace per (device, stream): scratch of the staged selection of rows longer than 8192 keys
# (no initialisation needed). Grown on demand, so steady-state calls allocate nothing.
_TOPK_WS: dict = {}


def _topk_workspace(dev: torch.device, stream: int, rows: int, n: int, k: int, nparts: int = 0):
    nbytes = int(_lib.load().dsv32_topk_workspace_bytes(rows, n, k, nparts))
    if nbytes < 0:
        _lib.check(-nbytes, "topk workspace")
    if nbytes == 0:
        return None, 0
    key = (dev.index, stream)
    ws = _TOPK_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        _TOPK_WS[key] = ws
    return ws.data_ptr(), ws.numel()


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("deepseek_v32_gtx1650_b200 kernels run on CUDA tensors only (no CPU path)")


def act_quant(x: torch.Tensor, round_scale: bool = False, block_m: int = 32):
    """x [..., N] -> (int8 [..., N], fp32 scales [..., N // 128]). kernels.py:55-64."""
    assert x.is_contiguous() and x.shape[-1] % GROUP == 0
    assert x.dtype in _DT, f"act_quant supports float32/bfloat16/float16, got {x.dtype}"
    _require_cuda(x)
    N = x.shape[-1]
    x2 = x.view(-1, N)
    M = x2.shape[0]
    NG = N // GROUP
    y = torch.empty_like(x2, dtype=torch.int8)
    s = torch.empty(M, NG, device=x.device, dtype=torch.float32)
    if M > 0 and N > 0:
        with _OnDevice(x):
            _lib.check(_lib.load().dsv32_act_quant(x2.data_ptr(), _DT[x.dtype], M, N, int(bool(round_scale)),
                                                   y.data_ptr(), s.data_ptr(), _stream(x)), "act_quant")
    return y.view(x.shape), s.view(*x.shape[:-1], NG)


def int8_gemm(a, a_s, b, b_s, out_dtype=torch.float32, version="v1"):
    """a [..., K] int8, a_s [..., K // 128], b [N, K] int8, b_s [N // 128, K // 128] -> [..., N].
    kernels.py:109-127."""
    assert a.is_contiguous() and b.is_contiguous() and a_s.is_contiguous() and b_s.is_contiguous()
    K = a.shape[-1]
    N = b.shape[0]
    M = a.numel() // K if K else 0
    KG = K // GROUP
    assert K % GROUP == 0 and N % GROUP == 0
    assert a.dtype == torch.int8 and b.dtype == torch.int8 and b.shape[1] == K
    assert a_s.dtype == torch.float32 and b_s.dtype == torch.float32
    assert a_s.numel() == M * KG and b_s.numel() == (N // GROUP) * KG
    assert out_dtype in _DT, f"unsupported out_dtype {out_dtype}"
    _require_cuda(a, a_s, b, b_s)
    c = torch.empty(*a.shape[:-1], N, device=a.device, dtype=out_dtype)
    if M > 0 and N > 0 and K > 0:
        with _OnDevice(a):
            st = _stream(a)
            ws, wsb = _gemm_workspace(a.device, st, M, N, K)
            _lib.check(_lib.load().dsv32_int8_gemm(a.data_ptr(), a_s.data_ptr(), b.data_ptr(), b_s.data_ptr(),
                                                   c.data_ptr(), _DT[out_dtype], M, N, K, ws, wsb, st), "int8_gemm")
    return c


def int8_gemm_partials(a, a_s, b, b_s):
    """Debug form of int8_gemm on the same tensor-core path: returns (c fp32 [M, N],
    partials int32 [K // 128, M, N]) where partials[kb] is the exact integer A_kb . B_kb^T."""
    assert a.is_contiguous() and b.is_contiguous() and a_s.is_contiguous() and b_s.is_contiguous()
    K = a.shape[-1]
    N = b.shape[0]
    M = a.numel() // K
    assert K % GROUP == 0 and N % GROUP == 0 and a.dtype == torch.int8 and b.dtype == torch.int8
    _require_cuda(a, a_s, b, b_s)
    c = torch.empty(M, N, device=a.device, dtype=torch.float32)
    p = torch.empty(K // GROUP, M, N, device=a.device, dtype=torch.int32)
    with _OnDevice(a):
        st = _stream(a)
        ws, wsb = _gemm_workspace(a.device, st, M, N, K)
        _lib.check(_lib.load().dsv32_int8_gemm_partials(a.data_ptr(), a_s.data_ptr(), b.data_ptr(), b_s.data_ptr(),
                                                        c.data_ptr(), p.data_ptr(), M, N, K, ws, wsb, st),
                   "int8_gemm_partials")
    return c, p


def _index_checks(q, w, k, k_s):
    assert q.dim() == 4 and k.dim() == 3, "q [b, m, h, d], k [b, n, d]"
    B, M, H, D = q.shape
    assert q.is_contiguous() and k.is_contiguous() and w.is_contiguous() and k_s.is_contiguous()
    assert k.shape[0] == B and k.shape[2] == D
    assert q.dtype == torch.int8 and k.dtype == torch.int8
    assert w.dtype == torch.float32 and k_s.dtype == torch.float32
    assert w.shape == (B, M, H) and k_s.shape == (B, k.shape[1])
    return B, M, H, D, k.shape[1]


def int8_index(q, w, k, k_s, causal=False, start=0, block_q=None, block_n=None, num_warps=None):
    """q [b, m, h, d] int8, w [b, m, h] fp32, k [b, n, d] int8, k_s [b, n] fp32 -> [b, m, n] fp32.
    causal: keys after start + m get -inf. kernels.py:165-178."""
    B, M, H, D, Nk = _index_checks(q, w, k, k_s)
    _require_cuda(q, w, k, k_s)
    o = torch.empty(B, M, Nk, device=q.device, dtype=torch.float32)
    if B and M and Nk:
        with _OnDevice(q):
            _lib.check(_lib.load().dsv32_int8_index(q.data_ptr(), w.data_ptr(), k.data_ptr(), k_s.data_ptr(),
                                                    o.data_ptr(), B, M, Nk, H, D, int(bool(causal)), int(start), 0,
                                                    _stream(q)), "int8_index")
    return o


def select_topk(scores: torch.Tensor, k: int, idx_offset: int = 0, cand_idx: torch.Tensor | None = None):
    """Top-k of every row of scores [..., n] fp32 -> (idx int32 [..., k], vals fp32 [..., k]).

    Replaces torch.topk on indexer scores. The k largest values are kept, ties at the k-th value
    go to the lowest positions, and results are listed in increasing position order (not by
    value). idx = position + idx_offset, or cand_idx[..., position] when cand_idx is given
    (merging candidate lists from key-range shards)."""
    assert scores.dtype == torch.float32 and scores.is_contiguous()
    n = scores.shape[-1]
    assert 1 <= k <= n, "k must be in [1, n]"
    _require_cuda(scores)
    rows = scores.numel() // n if n else 0
    idx = torch.empty(*scores.shape[:-1], k, device=scores.device, dtype=torch.int32)
    vals = torch.empty(*scores.shape[:-1], k, device=scores.device, dtype=torch.float32)
    if cand_idx is not None:
        assert cand_idx.dtype == torch.int32 and cand_idx.is_contiguous() and cand_idx.shape == scores.shape
        cp, cld = cand_idx.data_ptr(), n
    else:
        cp, cld = None, 0
    if rows:
        with _OnDevice(scores):
            st = _stream(scores)
            ws, wsb = _topk_workspace(scores.device, st, rows, n, k)
            _lib.check(_lib.load().dsv32_topk(scores.data_ptr(), rows, n, n, cp, cld, int(idx_offset), k,
                                              idx.data_ptr(), vals.data_ptr(), ws, wsb, st), "select_topk")
    return idx, vals


def _ptr_array(ptrs):
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    return ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)), arr


def topk_parts_raw(val_ptrs, id_ptrs, rows: int, part_ld: int, part_len: int, k: int, device: torch.device,
                   workspace=None, out=None):
    """Top-k over rows that are the concatenation of len(val_ptrs) lists given as raw device
    addresses (list j of row r at val_ptrs[j] + 4 * r * part_ld, ids likewise), which may be other
    GPUs' memory mapped with CUDA IPC. workspace: (device address, bytes) reserved by the caller
    (default: the per-stream top-k workspace); out: (idx, vals) tensors to write. Returns
    (idx int32 [rows, k], vals fp32 [rows, k])."""
    idx, vals = out if out is not None else (torch.empty(rows, k, device=device, dtype=torch.int32),
                                             torch.empty(rows, k, device=device, dtype=torch.float32))
    pv, keep_v = _ptr_array(val_ptrs)
    pi, keep_i = _ptr_array(id_ptrs)
    with _OnDevice(idx):
        st = _stream(idx)
        ws, wsb = workspace if workspace is not None else _topk_workspace(device, st, rows, len(val_ptrs) * part_len,
                                                                           k, len(val_ptrs))
        _lib.check(_lib.load().dsv32_topk_parts(pv, pi, len(val_ptrs), rows, part_ld, part_len, k, idx.data_ptr(),
                                                vals.data_ptr(), ws, wsb, st), "select_topk_parts")
    return idx, vals


def topk_parts_to_raw(val_ptrs, id_ptrs, rows: int, part_ld: int, part_len: int, k: int, out_idx_ptrs,
                      out_val_ptrs, device: torch.device, workspace=None):
    """topk_parts_raw writing every selected row to each (out_idx_ptrs[d], out_val_ptrs[d]) pair of raw
    [rows, k] device addresses (this GPU's or other GPUs' memory mapped with CUDA IPC) instead of
    returning it. The writes to other GPUs are complete when the kernel is; order them before the
    owners read (a collective)."""
    assert len(out_idx_ptrs) == len(out_val_ptrs) and 1 <= len(out_idx_ptrs) <= 16
    pv, keep_v = _ptr_array(val_ptrs)
    pi, keep_i = _ptr_array(id_ptrs)
    po, keep_o = _ptr_array(out_idx_ptrs)
    pw, keep_w = _ptr_array(out_val_ptrs)
    with torch.cuda.device(device):
        st = torch.cuda.current_stream(device).cuda_stream
        ws, wsb = workspace if workspace is not None else _topk_workspace(device, st, rows, len(val_ptrs) * part_len,
                                                                           k, len(val_ptrs))
        _lib.check(_lib.load().dsv32_topk_parts_to(pv, pi, len(val_ptrs), rows, part_ld, part_len, k, po, pw,
                                                   len(out_idx_ptrs), ws, wsb, st), "topk_parts_to")


def select_topk_parts(vals_list, idx_list, k: int):
    """Top-k of rows given as lists: row r of the concatenation of vals_list[j][r] (each [rows, L]
    fp32, L % 16 == 0) with candidate ids idx_list[j][r] (int32). The lists are read in place (no
    concatenation copy); selection and ties as select_topk. Returns (idx int32 [rows, k], vals)."""
    assert len(vals_list) == len(idx_list) and 1 <= len(vals_list) <= 16
    rows, L = vals_list[0].shape
    for v, i in zip(vals_list, idx_list):
        assert v.dtype == torch.float32 and i.dtype == torch.int32 and v.is_contiguous() and i.is_contiguous()
        assert v.shape == (rows, L) and i.shape == (rows, L) and v.device == vals_list[0].device
    _require_cuda(*vals_list, *idx_list)
    return topk_parts_raw([v.data_ptr() for v in vals_list], [i.data_ptr() for i in idx_list], rows, L, L, k,
                          vals_list[0].device)


def _index_topk_launch(q, w, k, k_s, n_keys, scores, scores_out, topk, causal, start, key_offset, out_idx_ptr,
                       out_val_ptr):
    B, M, H, D = q.shape
    lib = _lib.load()
    with _OnDevice(q):
        s = _stream(q)
        ws, wsb = _topk_workspace(q.device, s, B * M, n_keys, topk)
        _lib.check(lib.dsv32_int8_index_topk(q.data_ptr(), w.data_ptr(), k.data_ptr(), k_s.data_ptr(),
                                             scores.data_ptr(), B, M, n_keys, H, D, int(bool(causal)), int(start),
                                             k.shape[1], int(bool(scores_out)), topk, int(key_offset), out_idx_ptr,
                                             out_val_ptr, ws, wsb, s), "int8_index_topk")


def int8_index_topk(q, w, k, k_s, topk=2048, causal=False, start=0, return_scores=True, key_offset=0, n_keys=None):
    """Indexer scores + per-query top-k in one call (the step bench_indexer_e2e.py:54-57,72-77 runs).

    Returns (scores [b, m, n], idx int32 [b, m, topk], vals fp32 [b, m, topk]), or (idx, vals) when
    return_scores is False. idx are key positions (+ key_offset), in increasing order per query;
    see select_topk for the tie rule. n_keys: score only the first n_keys keys of each batch of k / k_s
    (a key cache [b, capacity, d] read in place); default all of them."""
    B, M, H, D, cap = _index_checks(q, w, k, k_s)
    Nk = cap if n_keys is None else int(n_keys)
    assert 1 <= Nk <= cap, "n_keys must be in [1, k.shape[1]]"
    assert 1 <= topk <= Nk, "topk must be in [1, n]"
    _require_cuda(q, w, k, k_s)
    scores = torch.empty(B, M, Nk, device=q.device, dtype=torch.float32)
    idx = torch.empty(B, M, topk, device=q.device, dtype=torch.int32)
    vals = torch.empty(B, M, topk, device=q.device, dtype=torch.float32)
    if B and M:
        _index_topk_launch(q, w, k, k_s, Nk, scores, return_scores, topk, causal, start, key_offset, idx.data_ptr(),
                           vals.data_ptr())
    return (scores, idx, vals) if return_scores else (idx, vals)


def int8_index_topk_into(q, w, k, k_s, out_idx_ptr: int, out_val_ptr: int, topk=2048, causal=False, start=0,
                         key_offset=0):
    """int8_index_topk writing the selection to raw device addresses ([b * m, topk] int32 ids and
    fp32 values, e.g. a buffer other GPUs map); the scores go to a temporary."""
    B, M, H, D, Nk = _index_checks(q, w, k, k_s)
    assert 1 <= topk <= Nk, "topk must be in [1, n]"
    _require_cuda(q, w, k, k_s)
    scores = torch.empty(B, M, Nk, device=q.device, dtype=torch.float32)
    if B and M:
        _index_topk_launch(q, w, k, k_s, Nk, scores, False, topk, causal, start, key_offset, out_idx_ptr,
                           out_val_ptr)


def rotate_quant(x: torch.Tensor, rotate: bool = True, scale_mul: torch.Tensor | None = None):
    """The indexer's operand producer: x [..., 128] fp32/bf16/fp16 -> (int8 [..., 128], fp32 [...]).
    Each 128-vector is rotated by the Hadamard transform scaled by 128^-1/2 (rotate=True) and
    quantised with one scale per vector (hadamard_quant.py:63-103), in the row-major layout
    int8_index reads. scale_mul (fp32, shape x.shape[:-1]): the scales come back multiplied by it,
    one fp32 rounding (the indexer's w * qs, bench_indexer_e2e.py:55)."""
    assert x.is_contiguous() and x.shape[-1] == GROUP, "rotate_quant works on 128-value vectors"
    assert x.dtype in _DT, f"rotate_quant supports float32/bfloat16/float16, got {x.dtype}"
    _require_cuda(x)
    rows = x.numel() // GROUP
    if scale_mul is not None:
        assert scale_mul.dtype == torch.float32 and scale_mul.is_contiguous()
        assert scale_mul.shape == x.shape[:-1] and scale_mul.device == x.device
    y = torch.empty(x.shape, device=x.device, dtype=torch.int8)
    s = torch.empty(x.shape[:-1], device=x.device, dtype=torch.float32)
    if rows:
        with _OnDevice(x):
            _lib.check(_lib.load().dsv32_rotate_quant(x.data_ptr(), _DT[x.dtype], rows, int(bool(rotate)),
                                                      y.data_ptr(), s.data_ptr(),
                                                      None if scale_mul is None else scale_mul.data_ptr(),
                                                      _stream(x)), "rotate_quant")
    return y, s


def weight_quant(w: torch.Tensor):
    """GEMM weight block quantiser: w [N, K] fp32/bf16/fp16 -> (int8 [N, K], fp32 [N // 128, K // 128]),
    one scale max(amax, 1e-4) / 127 per 128 x 128 block (test_kernels.py:80-82, bench.py:43-44)."""
    assert w.is_contiguous() and w.dim() == 2 and w.shape[0] % GROUP == 0 and w.shape[1] % GROUP == 0
    assert w.dtype in _DT, f"weight_quant supports float32/bfloat16/float16, got {w.dtype}"
    _require_cuda(w)
    N, K = w.shape
    wq = torch.empty(N, K, device=w.device, dtype=torch.int8)
    ws = torch.empty(N // GROUP, K // GROUP, device=w.device, dtype=torch.float32)
    if N and K:
        with _OnDevice(w):
            _lib.check(_lib.load().dsv32_weight_quant(w.data_ptr(), _DT[w.dtype], N, K, wq.data_ptr(), ws.data_ptr(),
                                                      _stream(w)), "weight_quant")
    return wq, ws
