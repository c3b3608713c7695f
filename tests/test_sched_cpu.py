"""The batching scheduler (ekv_sched_*) on a host-only pool against the scheduler model of
oracle/block_model.py: admission order, sequence ids and block tables, block reuse counts,
completion, and the pool's free list after every tick. No GPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "embodied.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import ekv  # noqa: E402
from block_model import PoolModel, SchedModel  # noqa: E402


def _host_pool(n_blocks, bt, max_seqs, max_bps):
    return ekv.Pool(device=-1, dtype=ekv.DTYPE_Q8_0, block_tokens=bt, n_blocks=n_blocks, kv_heads=1,
                    head_dim=256, n_layers=2, max_seqs=max_seqs, max_blocks_per_seq=max_bps, suffix_tokens=50)


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_scheduler_matches_model(seed):
    rng = np.random.default_rng(seed)
    bt, n_blocks, max_seqs, max_bps = 16, int(rng.integers(150, 400)), 12, 64
    max_batch, n_steps = int(rng.integers(3, 12)), int(rng.integers(1, 6))
    pool = _host_pool(n_blocks, bt, max_seqs, max_bps)
    sched = ekv.Scheduler(pool, max_batch, n_steps)
    mpool = PoolModel(n_blocks, bt, max_seqs, max_bps)
    msched = SchedModel(mpool, max_batch, n_steps)
    rid = 1000
    for tick in range(60):
        for _ in range(int(rng.integers(0, 4))):
            plen = int(rng.integers(0, 1100))
            pv = int(rng.integers(0, plen + 1))
            exp = msched.submit(rid, plen, pv)
            if exp == "ok":
                sched.submit(rid, plen, pv)
            else:
                with pytest.raises(ekv.EkvError) as e:
                    sched.submit(rid, plen, pv)
                assert e.value.code == ekv.ERR_RANGE
            rid += 1
        t = sched.begin_tick()
        m = msched.begin_tick()
        assert t.request_ids == m["request_ids"]
        assert t.seq_ids_host == m["seq_ids"]
        assert t.steps == m["steps"]
        assert t.admitted_index == m["admitted_index"]
        assert t.blocks_reused == m["blocks_reused"]
        assert t.queued == m["queued"]
        # host-only pool: the "device" arrays are host memory
        n = t.n_batch
        if n:
            arr = np.ctypeslib.as_array(ctypes_ptr(t.seq_ids.ptr), (n,))
            assert list(arr) == m["seq_ids"]
            pvs = np.ctypeslib.as_array(ctypes_ptr(t.prefix_valid.ptr), (n,))
            assert list(pvs) == m["prefix_valid"]
        na = len(t.admitted_index)
        if na:
            plens = np.ctypeslib.as_array(ctypes_ptr(t.admitted_prefix_len.ptr), (na,))
            assert list(plens) == [msched.active[i]["plen"] for i in m["admitted_index"]]
            assert t.max_admitted_prefix == max(plens)
            src = np.ctypeslib.as_array(ctypes_ptr(t.admitted_src_row.ptr), (na,))
            assert list(src) == list(np.concatenate([[0], np.cumsum(plens)[:-1]]))
            assert t.admitted_rows == int(np.sum(plens))
            zeros = np.ctypeslib.as_array(ctypes_ptr(t.admitted_zeros.ptr), (na,))
            assert not zeros.any()
            seqs = np.ctypeslib.as_array(ctypes_ptr(t.admitted_seq_ids.ptr), (na,))
            assert list(seqs) == [m["seq_ids"][i] for i in m["admitted_index"]]
        for s in m["seq_ids"]:
            v = pool.seq_get(s)
            assert v.blocks == mpool.seqs[s]["blocks"]
            assert v.n_tokens == mpool.seqs[s]["n"]
        assert sched.end_tick() == msched.end_tick()
        assert pool.info().free_blocks == len(mpool.free)
        st = sched.stats()
        assert st["completed"] == msched.completed
        assert st["blocks_reused"] == msched.reused
        assert st["active"] == len(msched.active)
    sched.close()
    assert pool.info().live_seqs == 0


def test_blocks_are_reused_after_completion():
    """A pool that holds two requests at a time serves six: later admissions take the blocks the
    finished requests gave back (lowest free first), and every block is reused."""
    pool = _host_pool(n_blocks=100, bt=16, max_seqs=4, max_bps=64)
    sched = ekv.Scheduler(pool, max_batch=4, n_steps=2)
    for r in range(6):
        sched.submit(r, 800)  # 50 blocks each: two fit
    seen, reused, done = [], 0, []
    for _ in range(6):
        t = sched.begin_tick()
        assert t.n_batch <= 2
        reused += t.blocks_reused
        seen.append(t.request_ids)
        done += sched.end_tick()
    assert done == list(range(6))
    assert seen == [[0, 1], [0, 1], [2, 3], [2, 3], [4, 5], [4, 5]]
    assert reused == 4 * 50
    assert sched.stats()["blocks_reused"] == 200
    assert pool.info().free_blocks == 100


def test_submit_validation():
    pool = _host_pool(n_blocks=100, bt=16, max_seqs=4, max_bps=8)
    with pytest.raises(ekv.EkvError):
        ekv.Scheduler(pool, max_batch=5, n_steps=2)  # more than the pool's sequence slots
    sched = ekv.Scheduler(pool, max_batch=4, n_steps=2)
    for bad in [(-1, 0), (10, 11)]:
        with pytest.raises(ekv.EkvError) as e:
            sched.submit(0, *bad)
        assert e.value.code == ekv.ERR_INVALID_ARG
    with pytest.raises(ekv.EkvError) as e:
        sched.submit(0, 8 * 16 + 1)  # wider than a block table
    assert e.value.code == ekv.ERR_RANGE


def ctypes_ptr(addr):
    import ctypes as C
    return C.cast(C.c_void_p(addr), C.POINTER(C.c_int32))
