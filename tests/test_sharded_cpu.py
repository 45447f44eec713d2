"""Multi-rank host logic of the sharded paths on CPU: two gloo ranks in spawned processes.

The indexer is split by key range; every rank scores its keys with the causal limit shifted by
its first key, keeps a local top-k with global key ids, and the lists are exchanged and merged
(all-to-all by query row when the rows split evenly, else all-gather). Here the per-rank compute
and the row selection are the CPU oracle; the sharding helpers (shard_range, the causal shift,
merge_candidates, gather_candidates, gather_columns) are the product's. The merged selection must equal the
single-process top-k exactly, for several world sizes and causal offsets. A rank that fails before
the collective must make its peer's collective fail (short timeout), not hang it.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from deepseek_v32_gtx1650_b200 import sharded as S
from deepseek_v32_gtx1650_b200 import workloads as W


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _merge_oracle(cand_idx, cand_val, k):
    """Oracle merge: top-k by (value desc, candidate position asc) -> candidate ids, in id order."""
    pos, vals = O.topk_ref(cand_val, k)
    ids = np.take_along_axis(cand_idx, pos, axis=-1)
    return ids, vals


def _oracle_select(cand_val, k, cand_idx):
    ids, vals = _merge_oracle(cand_idx.numpy(), cand_val.numpy(), k)
    return torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(vals.astype(np.float32))


def _index_worker(rank, world, port, M, N, k, causal, start, q):
    try:
        _init(rank, world, port)
        qi, w, keys, ks = W.index_inputs(1, M, N, seed=7)
        lo, hi = S.shard_range(N, world, rank)
        sc = O.int8_index_ref(qi.numpy(), w.numpy(), keys[:, lo:hi].numpy(), ks[:, lo:hi].numpy(), causal=causal,
                              start=S.local_causal_start(start, lo))[0].astype(np.float32)
        li, lv = O.topk_ref(sc, k)
        idx = torch.from_numpy((li + lo).astype(np.int32))
        val = torch.from_numpy(lv.astype(np.float32))
        mi, mv = (t.numpy() for t in S.merge_candidates(idx, val, k, merge=_oracle_select))
        full = O.int8_index_ref(qi.numpy(), w.numpy(), keys.numpy(), ks.numpy(), causal=causal,
                                start=start)[0].astype(np.float32)
        gi, gv = O.topk_ref(full, k)
        q.put((rank, bool(np.array_equal(mi, gi) and np.array_equal(mv, gv)), ""))
    except Exception as e:  # report, never hang the parent
        q.put((rank, False, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(target, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    return sorted(res)


# M = 12 splits evenly over 2, 3 and 4 ranks (all-to-all by row); M = 10 over 4 and M = 13 over 3
# do not (all-gather)
@pytest.mark.parametrize("world,M,causal,start", [(2, 12, False, 0), (2, 12, True, 700), (3, 12, True, 300),
                                                  (4, 12, True, 0), (4, 10, True, 500), (3, 13, False, 0)])
def test_key_sharded_topk_merge_equals_single_process(world, M, causal, start):
    N, k = 1024, 64
    res = _run(_index_worker, world, M, N, k, causal, start)
    assert all(ok for _, ok, _ in res), res


def _gemm_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        a, a_s, b, b_s = W.gemm_inputs_uniform(16, 128 * 2 * world, 256, seed=3)
        lo, hi = S.shard_range(b.shape[0], world, rank)
        c_loc = O.int8_gemm_ref(a.numpy(), a_s.numpy(), b[lo:hi].numpy(), b_s[lo // 128:hi // 128].numpy())
        full = S.gather_columns(torch.from_numpy(c_loc))
        ref = O.int8_gemm_ref(a.numpy(), a_s.numpy(), b.numpy(), b_s.numpy())
        q.put((rank, bool(np.array_equal(full.numpy(), ref)), ""))
    except Exception as e:
        q.put((rank, False, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_n_sharded_gemm_columns_gather():
    res = _run(_gemm_worker, 2)
    assert all(ok for _, ok, _ in res), res


def _failing_worker(rank, world, port, q):
    """Rank 1 fails before the collective; rank 0 must get an error within its timeout."""
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            raise RuntimeError("injected failure before the all-gather")
        idx = torch.zeros(2, 4, dtype=torch.int32)
        S.gather_candidates(idx, torch.zeros(2, 4))
        q.put((rank, False, "collective completed without the failed peer"))
    except Exception as e:
        q.put((rank, True, type(e).__name__))
    finally:
        if rank == 0 and dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def test_failed_rank_surfaces_as_error_not_hang():
    res = _run(_failing_worker, 2)
    assert [ok for _, ok, _ in res] == [True, True], res


def test_shard_range_covers_keys_on_tile_boundaries():
    for n in (1, 127, 128, 4096, 131072, 131073):
        for world in (1, 2, 3, 8):
            parts = [S.shard_range(n, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            for (a, b), (c, d) in zip(parts, parts[1:]):
                assert b == c and (a % 128 == 0 or a == n)
