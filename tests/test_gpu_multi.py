"""Sharded paths on 2 GPUs (skipped with fewer GPUs): the key-range sharded indexer + top-k merge
(peer-memory exchange through CUDA IPC when the rows split evenly, NCCL all-gather otherwise) equals
the single-GPU int8_index_topk exactly; the N-sharded GEMM gathers to the 1-GPU output."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        import deepseek_v32_gtx1650_b200 as D
        from deepseek_v32_gtx1650_b200 import sharded as S, workloads as W
        dev = torch.device("cuda", rank)
        k = 2048

        def index_case(M, seed, N=16384):
            start = N - M
            q_, w, keys, ks = W.index_inputs(1, M, N, seed=seed)
            lo, hi = S.shard_range(N, world, rank)
            idx, vals = S.sharded_index_topk(q_.to(dev), w.to(dev), keys[:, lo:hi].contiguous().to(dev),
                                             ks[:, lo:hi].contiguous().to(dev), lo, topk=k, causal=True, start=start)
            gi, gv = D.int8_index_topk(q_.to(dev), w.to(dev), keys.to(dev), ks.to(dev), topk=k, causal=True,
                                       start=start, return_scores=False)
            return torch.equal(idx, gi) and torch.equal(vals, gv)

        # 256 rows: peer-memory exchange (twice: the mapped lists are reused), 255 rows: NCCL all-gather;
        # 65536 keys: each rank's 32768-key rows take the long-row filter before the merge
        ok_index = (index_case(256, 11) and index_case(256, 12) and index_case(255, 13)
                    and index_case(256, 14, N=65536))
        a, a_s, b, b_s = W.gemm_inputs_uniform(256, 256 * world, 1024, seed=5)
        blo, bhi = S.shard_range(b.shape[0], world, rank)
        c_loc = S.sharded_int8_gemm(a.to(dev), a_s.to(dev), b[blo:bhi].contiguous().to(dev),
                                    b_s[blo // 128:bhi // 128].contiguous().to(dev))
        full = S.gather_columns(c_loc)
        ref = D.int8_gemm(a.to(dev), a_s.to(dev), b.to(dev), b_s.to(dev))
        ok_gemm = ((full - ref).abs().max() / ref.abs().max()).item() < 1e-5  # K splits may differ
        dist.barrier()
        q.put((rank, bool(ok_index), bool(ok_gemm), ""))
    except Exception as e:
        q.put((rank, False, False, repr(e)))
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def test_sharded_index_topk_and_gemm_on_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] and r[2] for r in res), res
