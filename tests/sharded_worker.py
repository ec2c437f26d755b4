"""Worker for the multi-rank tests (one process per rank, launched by
torch.distributed.run).  Modes:

  cpu-merge   gloo only, no GPU: each rank takes its row shard
              (knn_shard_range of the C ABI), searches it with the oracle,
              all-gathers the per-rank (distance, index) lists and merges
              them; the result must equal the oracle on the full dataset.
  cpu-lost    gloo only: rank 1 leaves before the collective; rank 0 must
              get an error from its all-gather within the short timeout
              instead of hanging.
  gpu         one GPU per rank: row shards built with global offsets,
              NCCL communicator attached, every rank searches and receives
              the merged global result, checked against the oracle;
              graph-replayed peer-exchange searches, a 200 ms skew between
              the ranks, and a missing peer (bounded wait, KNN_ETIMEOUT).
  gpu-exact   one GPU per rank: exact fp32 re-ranking on every shard (the
              merged result must equal the oracle on the unrounded rows
              byte for byte) and the inner-product metric, through the
              NVLink peer exchange and the NCCL all-gather.
Exit code 0 = pass.
"""
import datetime
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "cuvs-silicon_b200"))


def main():
    import torch
    import torch.distributed as dist

    mode = sys.argv[1]
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    timeout = datetime.timedelta(seconds=8 if mode == "cpu-lost" else 120)
    dist.init_process_group("gloo", timeout=timeout)

    import cuvs_b200 as E
    import oracle as O

    n, dim, nq = 20011, 72, 37
    base = O.gen_iid(n, dim, 101)
    queries = O.gen_iid(nq, dim, 102)
    b16, q16 = O.round_fp16(base), O.round_fp16(queries)
    lo, hi = E.shard_range(n, world, rank)

    if mode == "cpu-merge":
        for k in (1, 10, 50):
            li, ld = O.port_knn(b16[lo:hi], q16, k)
            li = np.where(li == O.NO_INDEX, li, li + lo).astype(np.uint32)
            gi = [torch.empty((nq, k), dtype=torch.int64) for _ in range(world)]
            gd = [torch.empty((nq, k), dtype=torch.float32) for _ in range(world)]
            dist.all_gather(gi, torch.from_numpy(li.astype(np.int64)))
            dist.all_gather(gd, torch.from_numpy(ld))
            lists_i = np.stack([g.numpy().astype(np.uint32) for g in gi], axis=1)
            lists_d = np.stack([g.numpy() for g in gd], axis=1)
            mi, md = O.merge_lists(lists_d, lists_i)
            fi, fd = O.port_knn(b16, q16, k)
            assert np.array_equal(mi, fi) and np.array_equal(md, fd), f"k={k}"
        dist.barrier()
        dist.destroy_process_group()
        return 0

    if mode == "cpu-lost":
        if rank == 1:
            os._exit(0)  # leaves between steps, nothing in flight
        try:
            dist.all_gather([torch.empty(4) for _ in range(world)], torch.zeros(4))
        except Exception as e:  # the loss is detected on the host
            print(f"rank 0 detected the lost peer: {type(e).__name__}", flush=True)
            return 0
        print("rank 0: collective completed without its peer", flush=True)
        return 1

    if mode == "gpu":
        torch.cuda.set_device(rank)
        obj = [E.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        with E.Index(rank) as idx:
            idx.build(base[lo:hi], row_offset=lo, total_rows=n)
            idx.attach_comm(obj[0], world, rank)
            for k in (1, 10, 100, 256):
                gi, gd = idx.search(queries, k)
                oi, od = O.port_knn(b16, q16, k, threads=4)
                par = O.check_parity(b16, q16, gi, gd, oi, od, 1e-3)
                assert par.ok, f"rank {rank} k={k}: {par.detail}"
            # stream-ordered path with device buffers: the first search runs
            # directly, the second is captured into a CUDA graph, the rest
            # replay it (the exchange epoch advances on the device)
            qd = torch.from_numpy(queries).cuda()
            ni = torch.empty((nq, 10), dtype=torch.int32, device="cuda")
            nd = torch.empty((nq, 10), dtype=torch.float32, device="cuda")
            ref_i, ref_d = idx.search(queries, 10)
            for _ in range(5):
                ni.zero_()
                idx.search_async(qd, 10, ni, nd)
                idx.sync()
                assert np.array_equal(ni.cpu().numpy().view(np.uint32), ref_i)
                assert np.array_equal(nd.cpu().numpy(), ref_d)
            # host-side skew between ranks within the peer timeout: rank 1
            # issues its search 200 ms after rank 0
            dist.barrier()
            if rank == 1:
                time.sleep(0.2)
            gi, gd = idx.search(queries, 10)
            assert np.array_equal(gi, ref_i) and np.array_equal(gd, ref_d)
            # the NCCL all-gather fallback gives the same bytes
            idx.set_peer_exchange(False)
            gi, gd = idx.search(queries, 10)
            assert np.array_equal(gi, ref_i) and np.array_equal(gd, ref_d)
            idx.set_peer_exchange(True)
            gi, gd = idx.search(queries, 10)
            assert np.array_equal(gi, ref_i) and np.array_equal(gd, ref_d)
            dist.barrier()
            # failure detection: rank 1 skips this search, so rank 0's final
            # merge waits for lists that never come; its bounded wait must
            # give up and report KNN_ETIMEOUT (the GPU stays usable).  2,048
            # queries make several waves of merge blocks: once one block has
            # recorded the timeout the others give up at once, so the error
            # comes back after about one bound, not one bound per wave.
            many = O.gen_iid(2048, dim, 103)
            idx.set_peer_timeout(0.5)
            dist.barrier()
            if rank == 0:
                t0 = time.perf_counter()
                try:
                    idx.search(many, 10)
                    print("rank 0: search without its peer did not time out", flush=True)
                    return 1
                except RuntimeError as e:
                    waited = time.perf_counter() - t0
                    assert "ETIMEOUT" in str(e), str(e)
                    assert waited < 1.5, f"timeout took {waited:.2f} s for a 0.5 s bound"
                    print(f"rank 0 detected the missing peer list after {waited:.2f} s",
                          flush=True)
                torch.cuda.synchronize()
            dist.barrier()
        dist.barrier()
        dist.destroy_process_group()
        return 0
    if mode == "gpu-exact":
        torch.cuda.set_device(rank)
        obj = [E.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        with E.Index(rank) as idx:
            idx.set_rerank(True)
            idx.build(base[lo:hi], row_offset=lo, total_rows=n)
            idx.attach_comm(obj[0], world, rank)
            for peer in (True, False):
                idx.set_peer_exchange(peer)
                for k in (1, 10, 100):
                    gi, gd = idx.search(queries, k)
                    oi, od = O.port_knn(base, queries, k, threads=4)
                    assert idx.rerank_stats()["uncertified"] == 0, f"rank {rank} k={k}"
                    assert np.array_equal(gi, oi) and np.array_equal(gd, od), \
                        f"rank {rank} k={k} peer={peer}"
        # a communicator id serves one communicator: a new one for this index
        obj = [E.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        with E.Index(rank) as idx:
            idx.build(base[lo:hi], metric=E.METRIC_INNER_PRODUCT, row_offset=lo, total_rows=n)
            idx.attach_comm(obj[0], world, rank)
            for peer in (True, False):
                idx.set_peer_exchange(peer)
                for k in (10, 64):
                    gi, gd = idx.search(queries, k)
                    oi, od = O.port_knn(b16, q16, k, threads=4, metric=1)
                    par = O.check_parity_ip(b16, q16, gi, gd, oi, od, 1e-3)
                    assert par.ok, f"rank {rank} k={k} peer={peer}: {par.detail}"
        dist.barrier()
        dist.destroy_process_group()
        return 0
    raise SystemExit(f"unknown mode {mode}")


if __name__ == "__main__":
    sys.exit(main())
