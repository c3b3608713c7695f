"""CPU-side checks of the C-ABI library: it loads without a GPU, exports every symbol that
include/ekv.h declares, validates arguments, and its host-side block bookkeeping follows the
reference allocation policy (oracle/block_model.py). No kernel is launched."""
import ctypes as C
import os
import random
import re

import pytest

import ekv
from block_model import PoolModel

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "ekv.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ekv_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported():
    decl = declared_symbols()
    assert len(decl) >= 20
    lib = C.CDLL(ekv.LIB_PATH)
    missing = [s for s in decl if not hasattr(lib, s)]
    assert not missing, missing
    assert sorted(ekv.EXPORTED) == decl


def test_version_and_errors():
    assert "sm_100a" in ekv.version()
    assert ekv.lib.ekv_strerror(ekv.ERR_POOL_EXHAUSTED).decode() == "pool exhausted"


def host_pool(**kw):
    cfg = dict(device=-1, dtype=ekv.DTYPE_Q8_0, block_tokens=16, n_blocks=40, kv_heads=1,
               head_dim=256, n_layers=2, max_seqs=6, max_blocks_per_seq=12, suffix_tokens=50)
    cfg.update(kw)
    return ekv.Pool(**cfg)


@pytest.mark.parametrize("bad", [dict(block_tokens=12), dict(head_dim=40), dict(head_dim=48, dtype=ekv.DTYPE_Q8_0),
                                 dict(dtype=5), dict(n_blocks=0), dict(suffix_tokens=-1)])
def test_pool_config_validation(bad):
    with pytest.raises(ekv.EkvError):
        host_pool(**bad)


def test_host_pool_allocation_matches_model():
    rng = random.Random(1234)
    pool = host_pool()
    model = PoolModel(40, 16, 6, 12)
    code = {"ok": ekv.OK, "no_seq": ekv.ERR_NO_SEQ, "range": ekv.ERR_RANGE,
            "exhausted": ekv.ERR_POOL_EXHAUSTED, "invalid": ekv.ERR_INVALID_ARG,
            "unsupported": ekv.ERR_UNSUPPORTED}
    for step in range(4000):
        op = rng.choice(["create", "free", "resize", "resize", "evict", "set", "append", "append", "clear_pred",
                         "restore"])
        live = sorted(model.seqs)
        if op == "create":
            want = model.seq_create()
            try:
                got = pool.seq_create()
            except ekv.EkvError as e:
                assert want is None and e.code == ekv.ERR_POOL_EXHAUSTED
                continue
            assert got == want
        elif op == "free" and live:
            s = rng.choice(live)
            model.seq_free(s)
            pool.seq_free(s)
        elif op == "resize" and live:
            s = rng.choice(live)
            n = rng.randint(0, 200)
            want = model.seq_resize(s, n)
            rc = ekv.lib.ekv_seq_resize(pool.h, s, n)
            assert rc == code[want], (step, op, want, rc)
        elif op == "evict" and live:
            s = rng.choice(live)
            n = rng.randint(0, 4)
            want = model.seq_evict_front(s, n)
            rc = ekv.lib.ekv_seq_evict_front(pool.h, s, n)
            assert rc == code[want], (step, op, want, rc)
        elif op == "set" and live:
            s = rng.choice(live)
            blocks = rng.sample(range(40), rng.randint(0, 6))
            n = rng.randint(0, 16 * len(blocks))
            want = model.seq_set_blocks(s, blocks, n)
            arr = (C.c_int32 * max(1, len(blocks)))(*blocks)
            rc = ekv.lib.ekv_seq_set_blocks(pool.h, s, arr, len(blocks), n)
            assert rc == code[want], (step, op, want, rc)
        elif op == "append" and live:
            s = rng.choice(live)
            n = rng.choice([rng.randint(0, 40), 16 * rng.randint(0, 3)])
            pred = rng.random() < 0.5
            want = model.seq_append_tokens(s, n, pred)
            rc = ekv.lib.ekv_seq_append_tokens(pool.h, s, n, 1 if pred else 0)
            assert rc == code[want], (step, op, want, rc)
        elif op == "clear_pred" and live:
            s = rng.choice(live)
            want = model.seq_clear_pred(s)
            rc = ekv.lib.ekv_seq_clear_pred(pool.h, s)
            assert rc == code[want], (step, op, want, rc)
        elif op == "restore" and live:
            s = rng.choice(live)
            n = rng.randint(0, 40)
            want = model.seq_restore(s, n)
            rc = ekv.lib.ekv_seq_restore(pool.h, s, n)
            assert rc == code[want], (step, op, want, rc)
        for s, q in model.seqs.items():
            v = pool.seq_get(s)
            assert v.n_tokens == q["n"] and v.blocks == q["blocks"], (step, s)
            assert pool.seq_get_pred(s) == q["pred"], (step, s)
        assert pool.info().free_blocks == len(model.free)
    pool.close()


def test_exhaustion_leaves_pool_unchanged():
    pool = host_pool(n_blocks=8)
    a = pool.seq_create()
    pool.seq_resize(a, 16 * 6)
    b = pool.seq_create()
    before = pool.info().free_blocks
    with pytest.raises(ekv.EkvError) as e:
        pool.seq_resize(b, 16 * 3)
    assert e.value.code == ekv.ERR_POOL_EXHAUSTED
    assert pool.info().free_blocks == before and pool.seq_get(b).blocks == []
    pool.seq_free(a)
    pool.seq_resize(b, 16 * 3)
    assert pool.seq_get(b).blocks == [0, 1, 2]  # freed blocks are reused lowest-first


def test_data_ops_refuse_host_only_pool():
    pool = host_pool()
    s = pool.seq_create()
    pool.seq_resize(s, 32)
    rc = ekv.lib.ekv_gather(pool.h, 0, s, 0, 4, 0, C.c_void_p(16), C.c_void_p(16), None)
    assert rc == ekv.ERR_UNSUPPORTED


def test_append_suffix_attention_validates_before_enqueueing():
    pool = host_pool()
    s = pool.seq_create()
    pool.seq_resize(s, 32)
    ids = C.c_void_p(16)
    prm = ekv.AttnParams(0, 1, 50, 8, 0.0625, 0, 0, 0, 0, 0, 50, ekv.DTYPE_BF16, 1, 0, ids.value,
                         None, None, None, None)
    f = ekv.lib.ekv_append_suffix_attention
    buf = C.c_void_p(1 << 20)
    assert f(pool.h, C.byref(prm), None, buf, buf, buf, None, 0, None) == ekv.ERR_INVALID_ARG
    assert f(pool.h, C.byref(prm), C.c_void_p((1 << 20) + 8), buf, buf, buf, None, 0, None) == ekv.ERR_INVALID_ARG
    prm.suffix_len = 51
    assert f(pool.h, C.byref(prm), buf, buf, buf, buf, None, 0, None) == ekv.ERR_RANGE
    prm.suffix_len, prm.layer = 50, 7
    assert f(pool.h, C.byref(prm), buf, buf, buf, buf, None, 0, None) == ekv.ERR_INVALID_ARG
    prm.layer, prm.q_heads = 0, 0
    assert f(pool.h, C.byref(prm), buf, buf, buf, buf, None, 0, None) == ekv.ERR_INVALID_ARG


def test_predicted_tokens_roll_back():
    """LingBotKVCache's predict -> clear_pred -> clean append (models/lingbot_va.cpp:8853-8886,
    8954-8966): the clean tokens take the predicted ones' positions and blocks."""
    pool = host_pool()
    s = pool.seq_create()
    pool.seq_append_tokens(s, 40)
    pool.seq_append_tokens(s, 30, pred=True)
    assert pool.seq_get_pred(s) == (40, 70)
    blocks = pool.seq_get(s).blocks
    pool.seq_clear_pred(s)
    assert pool.seq_get(s).n_tokens == 40 and pool.seq_get_pred(s) == (0, 0)
    pool.seq_append_tokens(s, 30)
    assert pool.seq_get(s).blocks == blocks  # same blocks, same positions
    # a predicted range inside the sequence leaves as whole blocks; unaligned ones are refused
    pool.seq_resize(s, 48)
    pool.seq_append_tokens(s, 32, pred=True)
    pool.seq_append_tokens(s, 5)
    before = pool.seq_get(s).blocks
    pool.seq_clear_pred(s)
    v = pool.seq_get(s)
    assert v.n_tokens == 53 and v.blocks == before[:3] + before[5:]
    pool.seq_append_tokens(s, 3, pred=True)
    pool.seq_append_tokens(s, 2)
    with pytest.raises(ekv.EkvError) as e:
        pool.seq_clear_pred(s)
    assert e.value.code == ekv.ERR_UNSUPPORTED
    pool.seq_restore(s, 5)  # the rollback of the last two updates takes the predicted tokens too
    assert pool.seq_get(s).n_tokens == 53 and pool.seq_get_pred(s) == (0, 0)
    pool.close()
