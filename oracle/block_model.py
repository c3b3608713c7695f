"""Reference model of the pool's block bookkeeping. TEST INFRASTRUCTURE ONLY.

Restates, at block granularity, the slot policy of LingBotKVCache
(models/lingbot_va.cpp:8793-8831 of Embodied.cpp):
  * free slots are handed out in ascending index order (`free` is built ascending, :8803-8805,
    and re-sorted after evictions, :8826; `slots.assign(free.begin(), ...)`, :8829);
  * when a window is full the oldest entries are evicted first (:8806-8825). In the paged pool
    each sequence's block table is ordered oldest-first, so oldest-chunk eviction drops blocks
    from the front of the table;
  * a request that cannot be satisfied changes nothing and reports failure (:8791-8792,
    :8827-8828);
  * predicted tokens (is_pred, :8853-8886) are rolled back by clear_pred (:8954-8966) and the last
    update by restore (:8946-8952). The slot store frees those slots and its next update takes the
    lowest free slots again, so the clean tokens land where the predicted ones were; the paged pool
    keeps one predicted range per sequence and truncates it (or, inside the sequence, drops its
    whole blocks), which gives the same key order.
Sequence slots follow the same lowest-free-first rule. Lengths are in tokens.
"""
from __future__ import annotations


class PoolModel:
    def __init__(self, n_blocks: int, block_tokens: int, max_seqs: int, max_blocks_per_seq: int):
        self.bt = block_tokens
        self.free = set(range(n_blocks))
        self.n_blocks = n_blocks
        self.max_bps = max_blocks_per_seq
        self.free_seqs = set(range(max_seqs))
        self.seqs: dict[int, dict] = {}

    def _need(self, n_tokens):
        return (n_tokens + self.bt - 1) // self.bt

    def seq_create(self):
        if not self.free_seqs:
            return None
        s = min(self.free_seqs)
        self.free_seqs.remove(s)
        self.seqs[s] = {"n": 0, "blocks": [], "pred": (0, 0)}
        return s

    def seq_free(self, s):
        if s not in self.seqs:
            return False
        self.free.update(self.seqs[s]["blocks"])
        del self.seqs[s]
        self.free_seqs.add(s)
        return True

    def seq_resize(self, s, n_tokens):
        if s not in self.seqs:
            return "no_seq"
        q = self.seqs[s]
        need = self._need(n_tokens)
        if need > self.max_bps:
            return "range"
        have = len(q["blocks"])
        if need > have:
            if len(self.free) < need - have:
                return "exhausted"
            for _ in range(need - have):
                b = min(self.free)
                self.free.remove(b)
                q["blocks"].append(b)
        else:
            self.free.update(q["blocks"][need:])
            del q["blocks"][need:]
        q["n"] = n_tokens
        self._clamp(q)
        return "ok"

    @staticmethod
    def _clamp(q):
        lo, hi = q["pred"]
        hi = min(hi, q["n"])
        lo = min(lo, hi)
        q["pred"] = (lo, hi) if hi > lo else (0, 0)

    def seq_append_tokens(self, s, n, pred):
        if s not in self.seqs:
            return "no_seq"
        if n < 0:
            return "invalid"
        q = self.seqs[s]
        old = q["n"]
        lo, hi = q["pred"]
        if pred and hi > lo and hi != old:
            return "unsupported"
        r = self.seq_resize(s, old + n)
        if r != "ok":
            return r
        if pred and n > 0:
            q["pred"] = (old if hi <= lo else lo, old + n)
        return "ok"

    def seq_clear_pred(self, s):
        if s not in self.seqs:
            return "no_seq"
        q = self.seqs[s]
        lo, hi = q["pred"]
        if hi <= lo:
            return "ok"
        if hi == q["n"]:
            q["pred"] = (0, 0)
            return self.seq_resize(s, lo)
        if lo % self.bt or hi % self.bt:
            return "unsupported"
        self.free.update(q["blocks"][lo // self.bt:hi // self.bt])
        del q["blocks"][lo // self.bt:hi // self.bt]
        q["n"] -= hi - lo
        q["pred"] = (0, 0)
        return "ok"

    def seq_restore(self, s, n):
        if s not in self.seqs:
            return "no_seq"
        q = self.seqs[s]
        if n < 0 or n > q["n"]:
            return "range"
        return self.seq_resize(s, q["n"] - n)

    def seq_evict_front(self, s, n):
        if s not in self.seqs:
            return "no_seq"
        q = self.seqs[s]
        if n < 0 or n > len(q["blocks"]):
            return "range"
        self.free.update(q["blocks"][:n])
        del q["blocks"][:n]
        q["n"] = max(0, q["n"] - n * self.bt)
        lo, hi = q["pred"]
        q["pred"] = (max(0, lo - n * self.bt), max(0, hi - n * self.bt))
        self._clamp(q)
        return "ok"

    def seq_set_blocks(self, s, blocks, n_tokens):
        if s not in self.seqs:
            return "no_seq"
        if len(blocks) > self.max_bps or self._need(n_tokens) > len(blocks):
            return "range"
        q = self.seqs[s]
        own = set(q["blocks"])
        if len(set(blocks)) != len(blocks) or any(b < 0 or b >= self.n_blocks for b in blocks):
            return "invalid"
        if any(b not in own and b not in self.free for b in blocks):
            return "exhausted"
        self.free.update(q["blocks"])
        q["blocks"] = list(blocks)
        self.free.difference_update(blocks)
        q["n"] = n_tokens
        q["pred"] = (0, 0)
        return "ok"


class SchedModel:
    """Reference model of the batching scheduler over PoolModel: requests queue first come first
    served; a tick admits from the head of the queue while a sequence slot and the request's prefix
    blocks are free (the head that does not fit waits, and so does everything behind it), then every
    active request runs one step; a request that has run n_steps frees its sequence. The reference
    serves one request per predict (serving/vla-server.cpp:240-523); this is the batched version."""

    def __init__(self, pool: PoolModel, max_batch: int, n_steps: int):
        self.pool, self.max_batch, self.n_steps = pool, max_batch, n_steps
        self.queue, self.active = [], []
        self.used = set()
        self.completed = self.reused = 0

    def submit(self, rid, prefix_len, prefix_valid):
        if self.pool._need(prefix_len) > min(self.pool.max_bps, self.pool.n_blocks):
            return "range"
        self.queue.append((rid, prefix_len, prefix_valid))
        return "ok"

    def begin_tick(self):
        for a in self.active:
            a["adm"] = False
        reused = 0
        while self.queue and len(self.active) < self.max_batch:
            rid, plen, pvalid = self.queue[0]
            s = self.pool.seq_create()
            if s is None:
                break
            if self.pool.seq_resize(s, plen) != "ok":
                self.pool.seq_free(s)
                break
            for b in self.pool.seqs[s]["blocks"]:
                reused += b in self.used
                self.used.add(b)
            self.queue.pop(0)
            self.active.append(dict(rid=rid, seq=s, step=0, plen=plen, pvalid=pvalid, adm=True))
        self.reused += reused
        return dict(request_ids=[a["rid"] for a in self.active], seq_ids=[a["seq"] for a in self.active],
                    steps=[a["step"] for a in self.active], prefix_valid=[a["pvalid"] for a in self.active],
                    admitted_index=[i for i, a in enumerate(self.active) if a["adm"]],
                    blocks_reused=reused, queued=len(self.queue))

    def end_tick(self):
        done, keep = [], []
        for a in self.active:
            a["step"] += 1
            if a["step"] < self.n_steps:
                keep.append(a)
            else:
                self.pool.seq_free(a["seq"])
                done.append(a["rid"])
                self.completed += 1
        self.active = keep
        return done
