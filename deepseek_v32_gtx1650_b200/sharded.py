"""Multi-GPU partitioning of the hot path, one process per GPU over torch.distributed (NCCL).

Only the two paths that shard naturally are partitioned:

- int8_gemm by N: rank r owns a contiguous range of whole 128-column weight blocks (its rows of
  B and b_s); A and a_s are replicated. The kernel needs no collective. gather_columns()
  optionally all-gathers the column slices into the full [M, N] output.
- The indexer by key range: rank r owns keys [lo, hi) of the key cache (lo a multiple of 128).
  It scores every query against its keys with the causal limit shifted by -lo and selects its
  local top-k (global key ids = lo + position). The lists are then merged by query row: each
  rank's selection lands in a buffer every rank maps with CUDA IPC (PeerLists), a one-element
  all-reduce orders all selections before any read, rank r merges its rows / world rows with the
  top-k kernel (reading the other ranks' lists in place over NVLink, or with two ranks after pulling
  the peer's into its own memory with the copy engines), which writes the merged rows into every
  rank's output buffer (dsv32_topk_parts_to), and a second one-element all-reduce orders every merge
  before any rank reads its output. When the rows do not split
  evenly or peer mappings are unavailable, merge_candidates does the exchange with NCCL
  all-to-alls (or an all-gather). Local lists are position-ordered and concatenated in rank order,
  so ties resolve to the lowest global key id exactly as in the single-GPU selection; the merged
  result is identical to it.

The reference has no multi-GPU code (single GTX 1650); these are the two exchange patterns its
hot path admits.
"""
from __future__ import annotations

import atexit
import ctypes

import torch
import torch.distributed as dist

from . import _lib
from . import kernels as K


def shard_range(n: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """Contiguous [lo, hi) of n items for `rank`, boundaries on multiples of `align` (the last
    shard takes the remainder). Shards are as equal as the alignment allows."""
    units = (n + align - 1) // align
    base, extra = divmod(units, world)
    lo_u = rank * base + min(rank, extra)
    hi_u = lo_u + base + (1 if rank < extra else 0)
    return min(n, lo_u * align), min(n, hi_u * align)


def local_causal_start(start: int, lo: int) -> int:
    """Causal limit for a key shard starting at global key `lo`: query m sees global keys
    n <= start + m, i.e. local keys j <= (start - lo) + m."""
    return start - lo


def gather_candidates(idx: torch.Tensor, vals: torch.Tensor, group=None):
    """All-gather per-rank top-k lists ([rows, k] int32 ids, [rows, k] fp32 values) and return
    the candidates of every row concatenated in rank order: ([rows, world*k] int32, fp32).
    One collective: ids and value bits travel together as int32."""
    world = dist.get_world_size(group)
    rows, k = idx.shape
    packed = torch.stack([idx, vals.view(torch.int32)]).contiguous().view(-1)  # [2 * rows * k]
    out = torch.empty(world * packed.numel(), dtype=torch.int32, device=packed.device)
    dist.all_gather_into_tensor(out, packed, group=group)  # concatenated form: NCCL and gloo
    cand = out.view(world, 2, rows, k).permute(1, 2, 0, 3).reshape(2, rows, world * k)  # rank 0's k, rank 1's k..
    return cand[0].contiguous(), cand[1].contiguous().view(torch.float32)


def _select(cand_val, topk, cand_idx):
    return K.select_topk(cand_val, topk, cand_idx=cand_idx)


def merge_candidates(idx: torch.Tensor, vals: torch.Tensor, topk: int, group=None, merge=None):
    """Merge per-rank top-k lists ([rows, k] int32 global ids, [rows, k] fp32 values; every rank
    holds the same rows) into the top-`topk` of each row over all ranks, returned on every rank as
    ([rows, topk] int32, [rows, topk] fp32). `merge(cand_val, topk, cand_idx)` selects over a row's
    candidates (default: the top-k kernel); it is a parameter so the exchange logic can be checked
    against a CPU selection.

    rows divisible by the world size: rows are split into equal blocks; two all-to-alls (ids, value
    bits) give each rank every rank's lists for its block, it merges them, and two all-gathers
    assemble the merged blocks. Otherwise every list is all-gathered and every rank merges all rows.
    Either way a row's candidates are the ranks' lists concatenated in rank order."""
    merge = merge or _select
    world = dist.get_world_size(group)
    rows, k = idx.shape
    if world == 1:
        return (idx, vals) if topk == k else merge(vals, topk, idx)
    if rows % world:
        cidx, cval = gather_candidates(idx, vals, group)
        return merge(cval, topk, cidx)
    r = rows // world
    ids_in = torch.empty(world * r * k, dtype=torch.int32, device=idx.device)
    bits_in = torch.empty(world * r * k, dtype=torch.int32, device=idx.device)
    dist.all_to_all_single(ids_in, idx.contiguous().view(-1), group=group)
    dist.all_to_all_single(bits_in, vals.contiguous().view(torch.int32).view(-1), group=group)
    # source-rank-major [world, r, k] -> per row, the ranks' lists in rank order [r, world * k]
    cidx = ids_in.view(world, r, k).permute(1, 0, 2).reshape(r, world * k)
    cval = bits_in.view(world, r, k).permute(1, 0, 2).reshape(r, world * k).view(torch.float32)
    mi, mv = merge(cval, topk, cidx)
    out_i = torch.empty(rows, topk, dtype=torch.int32, device=idx.device)
    out_b = torch.empty(rows, topk, dtype=torch.int32, device=idx.device)
    dist.all_gather_into_tensor(out_i, mi.contiguous(), group=group)
    dist.all_gather_into_tensor(out_b, mv.contiguous().view(torch.int32), group=group)
    return out_i, out_b.view(torch.float32)


class _RawCuda:
    """A device buffer this process does not own by torch (a dsv32_device_alloc allocation), described
    by the CUDA array interface so that torch.as_tensor views it without a copy."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def _raw_view(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    typestr = {torch.int32: "<i4", torch.float32: "<f4"}[dtype]
    with torch.cuda.device(device):
        return torch.as_tensor(_RawCuda(ptr, shape, typestr), device=device)


class PeerLists:
    """This rank's top-k lists of `rows` rows (ids [rows, k] int32, then values [rows, k] fp32) and its
    output rows (ids, then values, [rows, k] each), in one cudaMalloc allocation, and every peer's,
    mapped into this process with CUDA IPC: the merge kernel reads the other ranks' lists in place
    over NVLink and writes its merged row block into every rank's output rows. Built once per (rows,
    k, device, group) by a collective (all ranks construct it together); released at exit. The
    merge's top-k workspace (rows of world * k candidates longer than one register pass are selected
    in stages) is reserved here too, so a merge allocates nothing. `usable` is False on every rank if
    any rank could not allocate, export or map (the caller then exchanges through NCCL)."""

    _cache: dict = {}

    def __init__(self, rows: int, k: int, device: torch.device, group=None):
        lib = _lib.load()
        self.rows, self.k, self.world, self.rank = rows, k, dist.get_world_size(group), dist.get_rank(group)
        self.bases, self.opened, self.own = [], [], 0
        self.ws, self.ws_arg = None, (None, 0)
        ok = True
        with torch.cuda.device(device):
            nbytes = int(lib.dsv32_topk_workspace_bytes(rows // self.world, self.world * k, k, self.world))
            if nbytes > 0:
                try:
                    self.ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
                    self.ws_arg = (self.ws.data_ptr(), nbytes)
                except RuntimeError:
                    ok = False
            base = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
            if ok and lib.dsv32_device_alloc(rows * k * 16, ctypes.byref(base)) == _lib.DSV32_OK:
                self.own = base.value
                ok = lib.dsv32_ipc_export(base, handle) == _lib.DSV32_OK
            else:
                ok = False
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw if ok else b"", group=group)
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.bases.append(self.own)
                    continue
                peer = ctypes.c_void_p()
                if ok and h and lib.dsv32_ipc_open(ctypes.create_string_buffer(h, len(h)),
                                                   ctypes.byref(peer)) == _lib.DSV32_OK:
                    self.bases.append(peer.value)
                    self.opened.append(peer.value)
                else:
                    ok = False
                    self.bases.append(0)
            # every rank takes the same exchange path: usable only if every mapping succeeded everywhere
            t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
            self.usable = bool(t.item())
        if not self.usable:
            self.close()
        else:  # this rank's output rows as tensors (copied out after every merge)
            self.out_ids = _raw_view(self.out_ids_ptr(self.rank), (rows, k), torch.int32, device)
            self.out_vals = _raw_view(self.out_vals_ptr(self.rank), (rows, k), torch.float32, device)
            # (two ranks) the peer's lists of this rank's row block, pulled in by the copy engines before
            # the merge: [ids, value bits] x rank x (rows / world) x k
            self.stage = (torch.empty(2, self.world, rows // self.world, k, dtype=torch.int32, device=device)
                          if self.world == 2 else None)
        self.flag = torch.zeros(1, dtype=torch.int32, device=device)
        atexit.register(self.close)

    def ids_ptr(self, r: int, row0: int = 0) -> int:
        return self.bases[r] + 4 * row0 * self.k

    def vals_ptr(self, r: int, row0: int = 0) -> int:
        return self.bases[r] + 4 * (self.rows + row0) * self.k

    def out_ids_ptr(self, r: int, row0: int = 0) -> int:
        return self.bases[r] + 4 * (2 * self.rows + row0) * self.k

    def out_vals_ptr(self, r: int, row0: int = 0) -> int:
        return self.bases[r] + 4 * (3 * self.rows + row0) * self.k

    def close(self):
        lib = _lib.load()
        self.out_ids = self.out_vals = self.stage = None
        for p in self.opened:
            lib.dsv32_ipc_close(ctypes.c_void_p(p))
        self.opened = []
        if self.own:
            lib.dsv32_device_free(ctypes.c_void_p(self.own))
            self.own = 0
        self.ws, self.ws_arg = None, (None, 0)

    @classmethod
    def get(cls, rows: int, k: int, device: torch.device, group=None):
        key = (rows, k, device.index, id(group))
        if key not in cls._cache:
            cls._cache[key] = cls(rows, k, device, group)
        return cls._cache[key]


def _p2p_usable(rows: int, k: int, world: int, device: torch.device, group=None) -> bool:
    """Whether the peer-memory merge applies: NCCL ranks on GPUs, rows that split evenly, lists of a
    multiple of 16, and a selection plan for rows of world * k candidates read as lists (host-side
    arithmetic, identical on every rank, so every rank takes the same path)."""
    if not (device.type == "cuda" and dist.get_backend(group) == "nccl" and 1 < world <= 16 and rows % world == 0
            and k % 16 == 0):
        return False
    return int(_lib.load().dsv32_topk_workspace_bytes(rows // world, world * k, k, world)) >= 0


def _mark(events, name):
    """Profiling hook: with a list, record a timing event on the current stream after a stage."""
    if events is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        events.append((name, ev))


def sharded_index_topk(q, w, k_local, k_s_local, key_lo: int, topk: int = 2048, causal: bool = False,
                       start: int = 0, group=None, events: list | None = None):
    """Key-range sharded indexer + top-k. q [B, M, H, D], w [B, M, H] replicated; k_local [B, n_r, D],
    k_s_local [B, n_r] this rank's keys starting at global key key_lo. Returns (idx int32 [B, M, topk],
    vals fp32 [B, M, topk]) on every rank, identical to the single-GPU int8_index_topk.
    events: optional list; a (stage name, CUDA event) pair is appended after each stage (for
    per-stage timing; the events must not be used inside a graph capture)."""
    B, M = q.shape[:2]
    assert k_local.shape[1] >= topk, "each key shard must hold at least topk keys"
    world = dist.get_world_size(group)
    rows = B * M
    lstart = local_causal_start(start, key_lo)
    ex = PeerLists.get(rows, topk, q.device, group) if _p2p_usable(rows, topk, world, q.device, group) else None
    if ex is None or not ex.usable:  # (usable is decided collectively: every rank takes the same path)
        idx, vals = K.int8_index_topk(q, w, k_local, k_s_local, topk=topk, causal=causal, start=lstart,
                                      return_scores=False, key_offset=key_lo)
        _mark(events, "index+local_topk")
        midx, mval = merge_candidates(idx.view(rows, topk), vals.view(rows, topk), topk, group)
        _mark(events, "nccl_exchange+merge")
        return midx.view(B, M, topk), mval.view(B, M, topk)
    # Peer-memory exchange: the local selection writes straight into this rank's mapped buffer, a
    # one-element all-reduce orders every rank's selection before any read, the merge kernel reads
    # this rank's row block of every rank's lists in place over NVLink and writes the merged block
    # into every rank's output rows (plain stores to peer memory, no staging copy), and a second
    # all-reduce orders every rank's merge before any rank reads its output.
    K.int8_index_topk_into(q, w, k_local, k_s_local, ex.ids_ptr(ex.rank), ex.vals_ptr(ex.rank), topk=topk,
                           causal=causal, start=lstart, key_offset=key_lo)
    _mark(events, "index+local_topk")
    dist.all_reduce(ex.flag, group=group)
    _mark(events, "order_allreduce")
    r = rows // world
    r0 = ex.rank * r
    # With two ranks the peer's lists of this row block are pulled into this GPU's memory by the copy
    # engines first (one cudaMemcpyAsync per array, over NVLink) and the merge reads only local memory:
    # 2 GPUs 2.874 -> 2.801 ms. With more ranks the copies, which run one after another on the stream,
    # cost more than the merge kernel's own loads from the peers (4 GPUs 1.649 -> 1.726 ms, 8 GPUs
    # 1.127 -> 1.281 ms), so the merge reads the peer lists in place.
    pull = world == 2
    lib = _lib.load()
    st = torch.cuda.current_stream(q.device).cuda_stream
    nb = r * topk * 4
    vals_p, ids_p = [], []
    for j in range(world):
        if j == ex.rank or not pull:
            vals_p.append(ex.vals_ptr(j, r0))
            ids_p.append(ex.ids_ptr(j, r0))
            continue
        di, dv = ex.stage[0, j].data_ptr(), ex.stage[1, j].data_ptr()
        _lib.check(lib.dsv32_copy_async(di, ex.ids_ptr(j, r0), nb, st), "peer list copy")
        _lib.check(lib.dsv32_copy_async(dv, ex.vals_ptr(j, r0), nb, st), "peer list copy")
        vals_p.append(dv)
        ids_p.append(di)
    if pull:
        _mark(events, "pull_peer_lists")
    K.topk_parts_to_raw(vals_p, ids_p, r, topk, topk, topk, [ex.out_ids_ptr(j, r0) for j in range(world)],
                        [ex.out_vals_ptr(j, r0) for j in range(world)], q.device, workspace=ex.ws_arg)
    _mark(events, "merge_to_every_rank")
    # A rank passes this all-reduce only after every rank's merge kernel has run, so its output rows
    # are complete, and the next call may overwrite the lists (the next merge writes the outputs only
    # after the next ordering all-reduce, which follows this rank's copy below).
    dist.all_reduce(ex.flag, group=group)
    out_i = ex.out_ids.clone()
    out_v = ex.out_vals.clone()
    _mark(events, "done_allreduce+copy")
    return out_i.view(B, M, topk), out_v.view(B, M, topk)


def sharded_int8_gemm(a, a_s, b_local, b_s_local, out_dtype=torch.float32):
    """N-sharded block-scaled GEMM: this rank's output columns [M, n_r] from its weight rows."""
    return K.int8_gemm(a, a_s, b_local, b_s_local, out_dtype=out_dtype)


def gather_columns(c_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather equal-width column slices [M, n_r] into the full [M, world * n_r] output."""
    world = dist.get_world_size(group)
    M, nr = c_local.shape
    out = torch.empty(world * M, nr, dtype=c_local.dtype, device=c_local.device)
    dist.all_gather_into_tensor(out, c_local.contiguous(), group=group)
    return out.view(world, M, nr).permute(1, 0, 2).reshape(M, world * nr)
