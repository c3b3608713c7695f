"""One rank of the multi-rank dispatch test (launched by tests/test_dispatch_multirank.py).

Runs on the CPU over `gloo`. Rank 0 scatters the request table, and every rank builds a host-side
pool (device -1: block bookkeeping only, no kernels) for its share. It computes each request's
attention output with the CPU oracle from the request's own seed, then gathers the results to
rank 0, which writes them to `<out>/results.npz`. A rank given `--fail-rank r` raises before the
gather instead, so the test can check that the other rank's collective ends with an error rather
than waiting forever.
"""
import argparse
import os
import sys
from datetime import timedelta

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "embodied.cpp_b200"), os.path.join(ROOT, "oracle")):
    sys.path.insert(0, p)

import torch.distributed as dist  # noqa: E402

import dispatch  # noqa: E402
import ekv  # noqa: E402
import oracle  # noqa: E402

TQ, HQ, HKV, D, BT = 4, 2, 1, 32, 16


def request_inputs(r: dispatch.RequestDesc):
    g = np.random.default_rng(r.seed)
    lk = r.prefix_len + TQ
    q = g.standard_normal((1, TQ, HQ, D)).astype(np.float32) * 0.5
    k = g.standard_normal((1, lk, HKV, D)).astype(np.float32) * 0.5
    v = g.standard_normal((1, lk, HKV, D)).astype(np.float32) * 0.5
    return q, k, v


def request_output(r: dispatch.RequestDesc) -> np.ndarray:
    q, k, v = request_inputs(r)
    seqs = oracle.make_seqs([r.prefix_len], prefix_valid=[r.prefix_valid], n_suffix=TQ)
    return oracle.attention(q, k, v, seqs, oracle.make_mask(), 1.0 / np.sqrt(D), n_threads=1)[0]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--n-req", type=int, default=9)
    ap.add_argument("--policy", default="balanced")
    ap.add_argument("--fail-rank", type=int, default=-1)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))

    table = dispatch.make_requests(args.n_req, 5, 60, seed=7, padded=False) if rank == 0 else None
    mine = dispatch.scatter_requests(table, world, rank, args.policy)

    # this rank's pool holds exactly its own requests
    need = [(r.prefix_len + BT - 1) // BT for r in mine]
    pool = ekv.Pool(device=-1, dtype=ekv.DTYPE_BF16, block_tokens=BT, n_blocks=max(1, sum(need)),
                    kv_heads=HKV, head_dim=D, n_layers=1, max_seqs=max(1, len(mine)),
                    max_blocks_per_seq=max([1] + need), suffix_tokens=TQ)
    tables = {}
    for r in mine:
        s = pool.seq_create()
        pool.seq_resize(s, r.prefix_len)
        tables[r.req_id] = pool.seq_get(s)
    local = {r.req_id: request_output(r) for r in mine}

    if rank == args.fail_rank:
        raise SystemExit(3)  # leaves between steps: no collective of this rank is in flight
    merged = dispatch.gather_results(local, world, rank)
    t = dispatch.max_over_ranks(float(rank + 1))
    import torch

    # the bench's end-of-step tensor gather: every rank's [2, 3] result stacked on rank 0
    stacked = dispatch.gather_outputs(torch.full((2, 3), float(rank + 1)), world, rank)
    if rank == 0:
        np.savez(os.path.join(args.out, "results.npz"), max_t=t, stacked=stacked.numpy(),
                 **{f"r{k}": v for k, v in merged.items()})
    else:
        assert stacked is None
    with open(os.path.join(args.out, f"rank{rank}.txt"), "w") as f:
        f.write(" ".join(str(r.req_id) for r in mine) + "\n")
        for k, sv in sorted(tables.items()):
            f.write(f"{k} {sv.n_tokens} {' '.join(map(str, sv.blocks))}\n")
    pool.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
