"""Benchmark of the denoise-loop attention over a paged prefix KV cache (libekv.so on B200).

Default workload (the one the headline metric is quoted on):
  pi0.5-shaped action-expert attention loop, 18 layers x 10 flow-matching steps, batch 64
  independent requests per GPU, prefix KV stored as ggml Q8_0 in 16-token blocks with shuffled
  block tables, prefix lengths uniform 700..816, 50 suffix (action) tokens appended per
  layer-step as bf16 and attending bidirectionally, 8 query heads over 1 KV head, head_dim 256,
  scale 1/16, Q/K/V = bf16(N(0,1) * 0.5), fixed seed.

One step = one predict's hot path for the batch: append the prefix K/V of all 18 layers into
the pool (Q8_0 quantise-on-write), then for each of the 10 x 18 layer-steps append the 50-token
suffix into its slot and run the masked attention. A query-token is one suffix token (all its
heads) through one attention call, so a step is 64 * 50 * 180 query-tokens.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--config NAME]

Multi-GPU (torchrun, one rank per GPU): every rank runs its own 64 requests (weak scaling), no
collective on the data path; timing is the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "embodied.cpp_b200"))

import dispatch  # noqa: E402  (request assignment, scatter/gather, max over ranks)

METRIC = "denoise-attn query-tok/s"

CONFIGS = {
    # name: (dtype, batch, prefix lo, prefix hi, text padding, description)
    "pi05_q8_b64": dict(dtype="q8_0", batch=64, plo=700, phi=816, padded=False,
                        desc="pi0.5 Q8_0 paged prefix (16-token blocks, shuffled tables), batch 64, "
                             "prefix U[700,816], 18 layers x 10 steps, 50 suffix tokens, 8q/1kv x 256"),
    "pi05_bf16_b1": dict(dtype="bf16", batch=1, plo=816, phi=816, padded=True,
                         desc="pi0.5 bf16 prefix 816 = 768 image + 48 text (valid text U[20,48], rest "
                              "padding-masked), batch 1, 18 layers x 10 steps, 50 suffix, 8q/1kv x 256"),
    "serve_q8_b256": dict(dtype="q8_0", batch=256, plo=600, phi=1000, padded=False,
                          desc="pi0.5 Q8_0 serving sweep, batch 256 per GPU, prefix U[600,1000], "
                               "18 layers x 10 steps, 50 suffix, 8q/1kv x 256"),
}

# BASELINE configs 3 and 4 (parity shapes; measured by `--config groot_b128` / `lingbot_b1`)
OTHER_CONFIGS = {
    "groot_b128": dict(kind="groot", batch=128,
                       desc="GR00T-N1.7 DiT action head: 16 layers (even: cross-attention of 17 queries to a cached "
                            "300-token backbone K/V, image span [0,256) and text [256,300) masks alternating; odd: "
                            "self-attention among the 17), 4 denoise steps, 32 heads x 48 (MHA), bf16, batch 128"),
    "pi05_proj_b64": dict(kind="proj", batch=64,
                          desc="pi0.5 action-expert Q/K/V projection + RoPE NEOX per layer-step, K/V into the pool's "
                               "suffix slots: batch 64 x 50 tokens, hidden 1024, 8q/1kv x 256, 18 layers per step, "
                               "bf16 weights and activations, f32 accumulation"),
    "lingbot_b1": dict(kind="lingbot", batch=1,
                       desc="LingBot-VA rollout: 30 layers, 24 heads x 128 (MHA), 16 chunks of 1560 video tokens "
                            "appended to a paged bf16 cache (64-token blocks, chunk stride 1600), block-causal "
                            "window of 8 chunks with oldest-chunk eviction, one episode per GPU"),
}

N_LAYERS, N_STEPS, TQ, HQ, HKV, D, BT = 18, 10, 50, 8, 1, 256, 16
SCALE = 1.0 / 16.0


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return dict(hbm=j["hbm_gbs"], tc=j["bf16_tflops"], tc_sustained=j.get("bf16_tflops_sustained"),
                    source="measured")
    return dict(hbm=6650.0, tc=1590.0, tc_sustained=1400.0, source="fallback")


# ------------------------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ------------------------------------------------------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------
# workload
# ------------------------------------------------------------------------------------------
class Pi05Workload:
    """Inputs of the pi0.5 denoise loop for `batch` requests, resident in HBM."""

    def __init__(self, cfg: dict, reqs, device: int):
        """`reqs`: this rank's request descriptors (dispatch.RequestDesc), already assigned."""
        import torch
        import ekv

        self.torch, self.ekv = torch, ekv
        self.cfg = cfg
        self.B = len(reqs)
        self.req_ids = [r.req_id for r in reqs]
        self.dtype = ekv.DTYPE_Q8_0 if cfg["dtype"] == "q8_0" else ekv.DTYPE_BF16
        seed = reqs[0].seed
        rng = np.random.default_rng(seed)
        B = self.B
        self.plen = np.array([r.prefix_len for r in reqs], np.int32)
        # pi0.5 bf16: 768 image tokens + 48 text slots, valid text U[20, 48], the rest padding-masked
        self.pvalid = np.array([r.prefix_valid for r in reqs], np.int32)
        need = (self.plen + BT - 1) // BT
        n_blocks = int(need.sum())
        self.pool = ekv.Pool(device=device, dtype=self.dtype, block_tokens=BT, n_blocks=n_blocks, kv_heads=HKV,
                             head_dim=D, n_layers=N_LAYERS, max_seqs=B, max_blocks_per_seq=int(need.max()),
                             suffix_tokens=TQ)
        perm = rng.permutation(n_blocks)
        self.seqs, o = [], 0
        for b in range(B):
            s = self.pool.seq_create()
            self.pool.seq_set_blocks(s, [int(x) for x in perm[o:o + need[b]]], int(self.plen[b]))
            o += int(need[b])
            self.seqs.append(s)
        self.pool.sync()
        dev = f"cuda:{device}"
        t = lambda a: torch.tensor(np.asarray(a, np.int32), device=dev)
        self.seq_ids = t(self.seqs)
        self.zeros = t(np.zeros(B))
        self.n_rows = t(self.plen)
        self.src_row = t(np.concatenate([[0], np.cumsum(self.plen)[:-1]]))
        self.prefix_valid = t(self.pvalid)
        self.total_rows = int(self.plen.sum())
        g = torch.Generator(device=dev).manual_seed(seed)
        rn = lambda *shape: (torch.randn(shape, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        n_calls = N_LAYERS * N_STEPS
        self.n_calls = n_calls
        # prefix K/V per layer (packed rows), per-call suffix K/V and Q, per-call output
        self.pk = rn(N_LAYERS, self.total_rows, HKV, D)
        self.pv = rn(N_LAYERS, self.total_rows, HKV, D)
        self.sk = rn(n_calls, B, TQ, HKV, D)
        self.sv = rn(n_calls, B, TQ, HKV, D)
        self.q = rn(n_calls, B, TQ, HQ, D)
        self.out = torch.empty((n_calls, B, TQ, HQ, D), dtype=torch.bfloat16, device=dev)
        self.params = [self.pool.attention_params(layer=l, seq_ids=self.seq_ids, q_tokens=TQ, q_heads=HQ,
                                                  scale=SCALE, suffix_len=TQ, out_dtype=ekv.DTYPE_BF16,
                                                  prefix_valid=self.prefix_valid)
                       for l in range(N_LAYERS)]
        ws = max(self.pool.workspace_size(p) for p in self.params)
        self.ws = torch.empty(ws, dtype=torch.uint8, device=dev) if ws else None
        # algorithmic work per call (masked / padded keys excluded)
        lk = (self.pvalid + TQ).astype(np.float64)
        self.flop_per_call = float((4.0 * TQ * HQ * lk * D).sum())
        b_kv = 34.0 / 32.0 if self.dtype == ekv.DTYPE_Q8_0 else 2.0
        self.bytes_per_call = float((TQ * HQ * D * 2 + 2 * HKV * self.pvalid * D * b_kv + 2 * HKV * TQ * D * 2
                                     + TQ * HQ * D * 2).sum())
        self.qtok_per_step = B * TQ * n_calls

    def step_prefix(self, stream):
        """Enqueue the step's prefix part: the 18 layers' prefix K/V into the pool."""
        for l in range(N_LAYERS):
            self.pool.append(l, self.seq_ids, self.zeros, self.n_rows, self.src_row, int(self.plen.max()), self.pk[l],
                             self.pv[l], stream=stream)

    def step_calls(self, stream):
        """Enqueue the step's 180 layer-step calls (ekv_append_suffix_attention: this step's suffix
        K/V and the attention over prefix + suffix)."""
        for c in range(self.n_calls):
            self.pool.append_suffix_attention(self.params[c % N_LAYERS], self.sk[c], self.sv[c], self.q[c], self.out[c],
                                              workspace=self.ws, stream=stream)

    def step(self, stream):
        self.step_prefix(stream)
        self.step_calls(stream)



# ------------------------------------------------------------------------------------------
# BASELINE configs 3 (GR00T) and 4 (LingBot): parity shapes, timed with the same contract
# ------------------------------------------------------------------------------------------
class GrootWorkload:
    """GR00T DiT action head over a cached backbone: per step, 16 layer-calls x 4 denoise steps;
    even layers cross-attend 17 queries to the layer's 300-token backbone K/V (image span or text
    mask, alternating), odd layers self-attend among the 17 (their K/V passed with the call)."""
    L, STEPS, T, H, DH, P, IMG = 16, 4, 17, 32, 48, 300, 256
    graphable = True

    def __init__(self, B, device):
        import torch
        import ekv
        self.ekv, self.B = ekv, B
        self.dtype = ekv.DTYPE_BF16
        L, T, H, DH, P = self.L, self.T, self.H, self.DH, self.P
        need = (P + 15) // 16
        self.pool = ekv.Pool(device=device, dtype=self.dtype, block_tokens=16, n_blocks=B * need, kv_heads=H,
                             head_dim=DH, n_layers=L, max_seqs=B, max_blocks_per_seq=need, suffix_tokens=T)
        self.seqs = []
        for _ in range(B):
            s = self.pool.seq_create()
            self.pool.seq_resize(s, P)
            self.seqs.append(s)
        self.pool.sync()
        dev = f"cuda:{device}"
        t = lambda a: torch.tensor(np.asarray(a, np.int32), device=dev)
        self.seq_ids = t(self.seqs)
        self.zeros, self.n_rows = t(np.zeros(B)), t(np.full(B, P))
        self.src_row = t(np.arange(B) * P)
        g = torch.Generator(device=dev).manual_seed(3)
        rn = lambda *shape: (torch.randn(shape, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        self.n_calls = L * self.STEPS
        self.pk, self.pv = rn(L // 2, B * P, H, DH), rn(L // 2, B * P, H, DH)
        self.sk, self.sv = rn(self.n_calls, B, T, H, DH), rn(self.n_calls, B, T, H, DH)
        self.q = rn(self.n_calls, B, T, H, DH)
        self.out = torch.empty((self.n_calls, B, T, H, DH), dtype=torch.bfloat16, device=dev)
        span_b, span_e = t(np.zeros(B)), t(np.full(B, self.IMG))
        self.params = []
        flop = byts = 0.0
        for l in range(L):
            if l % 2 == 0:
                flag = ekv.MASK_SPAN_ONLY if l % 4 == 0 else ekv.MASK_SPAN_EXCLUDE
                keys = self.IMG if flag == ekv.MASK_SPAN_ONLY else P - self.IMG
                self.params.append(self.pool.attention_params(layer=l, seq_ids=self.seq_ids, q_tokens=T, q_heads=H,
                                                              scale=DH ** -0.5, mask_flags=flag, span_begin=span_b,
                                                              span_end=span_e, out_dtype=ekv.DTYPE_BF16))
            else:
                keys = T
                self.params.append(self.pool.attention_params(layer=l, seq_ids=self.seq_ids, q_tokens=T, q_heads=H,
                                                              scale=DH ** -0.5, suffix_len=T, use_prefix=False,
                                                              out_dtype=ekv.DTYPE_BF16))
            flop += 4.0 * B * T * H * keys * DH
            byts += B * (2 * T * H * DH * 2 + 2 * keys * H * DH * 2)  # Q + O, visible K/V
        self.flop_per_call = flop / L
        self.bytes_per_call = byts / L
        self.qtok_per_step = B * T * self.n_calls
        self.ws = None

    def step_prefix(self, stream):
        for c in range(self.L // 2):  # the cross layers' backbone K/V
            self.pool.append(2 * c, self.seq_ids, self.zeros, self.n_rows, self.src_row, self.P, self.pk[c],
                             self.pv[c], stream=stream)

    def step_calls(self, stream):
        for c in range(self.n_calls):
            l = c % self.L
            if l % 2 == 0:
                self.pool.attention(self.params[l], self.q[c], self.out[c], stream=stream)
            else:
                self.pool.append_suffix_attention(self.params[l], self.sk[c], self.sv[c], self.q[c], self.out[c],
                                                  stream=stream)


class LingbotWorkload:
    """LingBot-VA world-action rollout for one episode: per step, 16 chunks; per chunk the window
    slides (oldest chunk evicted once 8 are held), then each of 30 layers appends the chunk's 1560
    K/V rows and attends the chunk's queries over the window (block-causal)."""
    L, CHUNKS, CT, STRIDE, WIN, H, DH = 30, 16, 1560, 1600, 8, 24, 128
    graphable = False  # the window moves on the host between chunks

    def __init__(self, B, device):
        import torch
        import ekv
        assert B == 1, "one episode per GPU"
        self.ekv, self.B = ekv, B
        self.dtype = ekv.DTYPE_BF16
        blocks_per_chunk = self.STRIDE // 64
        self.bpc = blocks_per_chunk
        self.pool = ekv.Pool(device=device, dtype=self.dtype, block_tokens=64,
                             n_blocks=(self.WIN + 1) * blocks_per_chunk, kv_heads=self.H, head_dim=self.DH,
                             n_layers=self.L, max_seqs=1, max_blocks_per_seq=(self.WIN + 1) * blocks_per_chunk,
                             suffix_tokens=0)
        self.seq = self.pool.seq_create()
        dev = f"cuda:{device}"
        t = lambda a: torch.tensor(np.asarray(a, np.int32), device=dev)
        self.seq_ids = t([self.seq])
        self.n_rows, self.src_row = t([self.CT]), t([0])
        self.dst = [t([w * self.STRIDE]) for w in range(self.WIN)]
        g = torch.Generator(device=dev).manual_seed(4)
        rn = lambda *shape: (torch.randn(shape, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        # per (chunk, layer) K/V and Q would be 16 x 30 x 3 x 9.6 MB; 4 distinct sets cycle (> L2)
        self.NSET = 4
        self.k = rn(self.NSET, self.L, self.CT, self.H, self.DH)
        self.v = rn(self.NSET, self.L, self.CT, self.H, self.DH)
        self.q = rn(self.NSET, self.L, self.CT, self.H, self.DH)
        self.out = torch.empty((self.NSET, self.L, self.CT, self.H, self.DH), dtype=torch.bfloat16, device=dev)
        self.params = [[self.pool.attention_params(layer=l, seq_ids=self.seq_ids, q_tokens=self.CT, q_heads=self.H,
                                                   scale=self.DH ** -0.5, mask_flags=ekv.MASK_BLOCK_CAUSAL,
                                                   chunk_tokens=self.CT, chunk_stride=self.STRIDE,
                                                   window_chunks=self.WIN, q_chunk0=w, out_dtype=ekv.DTYPE_BF16)
                        for l in range(self.L)] for w in range(self.WIN)]
        ws = max(self.pool.workspace_size(p) for p in self.params[self.WIN - 1])
        self.ws = torch.empty(ws, dtype=torch.uint8, device=dev) if ws else None
        self.n_calls = self.CHUNKS * self.L
        flop = 0.0
        for c in range(self.CHUNKS):
            held = min(c, self.WIN - 1) + 1
            flop += self.L * 4.0 * self.CT * self.H * (held * self.CT) * self.DH
        self.flop_per_call = flop / self.n_calls
        self.bytes_per_call = 0.0
        for c in range(self.CHUNKS):
            held = min(c, self.WIN - 1) + 1
            self.bytes_per_call += self.L * (2 * self.CT * self.H * self.DH * 2 + 2 * held * self.CT * self.H * self.DH * 2)
        self.bytes_per_call /= self.n_calls
        self.qtok_per_step = self.CT * self.n_calls

    def step_prefix(self, stream):
        self.pool.seq_resize(self.seq, 0)  # a fresh episode
        self.pool.sync(stream)

    def step_calls(self, stream):
        for c in range(self.CHUNKS):
            held = min(c, self.WIN - 1) + 1
            if c >= self.WIN:
                self.pool.seq_evict_front(self.seq, self.bpc)
            self.pool.seq_resize(self.seq, held * self.STRIDE)
            self.pool.sync(stream)
            w = held - 1
            for l in range(self.L):
                i = (c * self.L + l) % self.NSET
                self.pool.append(l, self.seq_ids, self.dst[w], self.n_rows, self.src_row, self.CT, self.k[i, l],
                                 self.v[i, l], stream=stream)
                self.pool.attention(self.params[w][l], self.q[i, l], self.out[i, l], workspace=self.ws, stream=stream)


class ProjWorkload:
    """The expert's per-layer-step Q/K/V projection with RoPE (ekv_project_qkv_rope) on the pi0.5 shape: 64
    requests x 50 action tokens, hidden 1024, 8 query heads and 1 KV head of 256, RoPE base 10000 at positions
    n_prefix + i, K/V written into the pool's suffix slots. One step = one denoise step (18 layer-steps, each
    with its own bf16 weights). Random-init weights N(0, 1/hidden), activations N(0,1) x 0.5."""
    L, T, HID, HQ, HKV, D = 18, 50, 1024, 8, 1, 256
    graphable = True

    def __init__(self, B, device):
        import torch
        import ekv
        self.ekv, self.B = ekv, B
        L, T, HID, HQ, HKV, D = self.L, self.T, self.HID, self.HQ, self.HKV, self.D
        self.pool = ekv.Pool(device=device, dtype=ekv.DTYPE_Q8_0, block_tokens=16, n_blocks=B, kv_heads=HKV,
                             head_dim=D, n_layers=L, max_seqs=B, max_blocks_per_seq=1, suffix_tokens=T)
        self.seqs = [self.pool.seq_create() for _ in range(B)]
        self.pool.sync()
        dev = f"cuda:{device}"
        self.seq_ids = torch.tensor(np.asarray(self.seqs, np.int32), device=dev)
        g = torch.Generator(device=dev).manual_seed(5)
        rn = lambda sc, *shape: (torch.randn(shape, generator=g, device=dev) * sc).to(torch.bfloat16)
        ws = HID ** -0.5
        self.wq, self.wk, self.wv = rn(ws, L, HQ * D, HID), rn(ws, L, HKV * D, HID), rn(ws, L, HKV * D, HID)
        self.x = rn(0.5, L, B * T, HID)  # > L2 together with the weights and outputs per step
        rng = np.random.default_rng(5)
        plens = rng.integers(700, 817, size=B)
        self.pos = torch.tensor(np.concatenate([np.arange(T) + p for p in plens]).astype(np.int32), device=dev)
        self.q = torch.empty((L, B, T, HQ, D), dtype=torch.bfloat16, device=dev)
        self.n_calls = L
        self.flop_per_call = 2.0 * B * T * (HQ + 2 * HKV) * D * HID
        self.bytes_per_call = 2.0 * (B * T * HID + (HQ + 2 * HKV) * D * HID + B * T * (HQ + 2 * HKV) * D)
        self.qtok_per_step = B * T * L
        self.ws = None

    def step_prefix(self, stream):
        pass

    def step_calls(self, stream):
        for l in range(self.L):
            self.ekv.project_qkv_rope(self.pool, l, self.seq_ids, self.x[l], self.wq[l], self.wk[l], self.wv[l],
                                      self.pos, 10000.0, self.q[l], tokens=self.T, q_heads=self.HQ, stream=stream)


class ServeWorkload:
    """a stream of pi0.5-shaped Q8_0 requests (prefix U[600, 1000], 50 action
    tokens, 10 denoise steps, 18 layers) served by the library's batching scheduler (ekv_sched_*)
    over one pool sized to `pool_gb` GB. Requests arrive at 256 / 10 per tick (a tick = one denoise
    step of every active request = 18 ekv_append_suffix_attention calls over the whole batch, plus
    the prefix appends of the requests admitted in it), so that in steady state 256 requests are
    active, about 26 complete per tick and the ones admitted next take the blocks they gave back
    (lowest free first). One bench step = 10 ticks (the work of one batch-256 predict)."""

    NSET = 36  # distinct per-call input sets (two ticks' worth, > L2), cycled

    def __init__(self, cfg, seed, device, pool_gb):
        import torch
        import ekv
        self.torch, self.ekv = torch, ekv
        self.B, self.plo, self.phi = cfg["batch"], cfg["plo"], cfg["phi"]
        self.rng = np.random.default_rng(seed)
        row_q8 = HKV * D // 32 * 34
        self.block_bytes_all_layers = N_LAYERS * 2 * BT * row_q8
        self.n_blocks = int(pool_gb * 1e9 // self.block_bytes_all_layers)
        self.pool_gb = pool_gb
        self.pool = ekv.Pool(device=device, dtype=ekv.DTYPE_Q8_0, block_tokens=BT, n_blocks=self.n_blocks,
                             kv_heads=HKV, head_dim=D, n_layers=N_LAYERS, max_seqs=self.B,
                             max_blocks_per_seq=(self.phi + BT - 1) // BT, suffix_tokens=TQ)
        self.sched = ekv.Scheduler(self.pool, self.B, N_STEPS)
        dev = f"cuda:{device}"
        g = torch.Generator(device=dev).manual_seed(seed)
        rn = lambda *shape: (torch.randn(shape, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        self.src_rows = 64 * self.phi  # admissions of one tick, packed
        self.pk = rn(N_LAYERS, self.src_rows, HKV, D)
        self.pv = rn(N_LAYERS, self.src_rows, HKV, D)
        self.sk = rn(self.NSET, self.B, TQ, HKV, D)
        self.sv = rn(self.NSET, self.B, TQ, HKV, D)
        self.q = rn(self.NSET, self.B, TQ, HQ, D)
        self.out = torch.empty((self.NSET, self.B, TQ, HQ, D), dtype=torch.bfloat16, device=dev)
        self.ws = None
        self.next_id, self.tick_no, self.call_no = 0, 0, 0
        self.pvalid = {}

    def arrivals(self):
        k = self.tick_no
        n = (self.B * (k + 1)) // N_STEPS - (self.B * k) // N_STEPS
        for _ in range(n):
            plen = int(self.rng.integers(self.plo, self.phi + 1))
            self.sched.submit(self.next_id, plen, plen)
            self.pvalid[self.next_id] = plen
            self.next_id += 1

    def tick(self, stream, ev=None):
        """Enqueue one tick; returns its counts. `ev` (start, end) brackets the 18 attention calls."""
        ekv = self.ekv
        self.arrivals()
        t = self.sched.begin_tick(stream)
        if t.admitted_index:
            if t.admitted_rows > self.src_rows:
                raise RuntimeError("admissions of one tick exceed the packed source rows")
            for l in range(N_LAYERS):
                self.pool.append(l, t.admitted_seq_ids, t.admitted_zeros, t.admitted_prefix_len, t.admitted_src_row,
                                 t.max_admitted_prefix, self.pk[l], self.pv[l], stream=stream)
        n = t.n_batch
        prms = [self.pool.attention_params(layer=l, seq_ids=t.seq_ids, q_tokens=TQ, q_heads=HQ, scale=SCALE,
                                           suffix_len=TQ, out_dtype=ekv.DTYPE_BF16, prefix_valid=t.prefix_valid)
                for l in range(N_LAYERS)]
        need = max(self.pool.workspace_size(p) for p in prms) if n else 0
        if need and (self.ws is None or self.ws.numel() < need):
            self.ws = self.torch.empty(need, dtype=self.torch.uint8, device=self.q.device)
        if ev is not None:
            ev[0].record(stream)
        for l in range(N_LAYERS):
            c = self.call_no % self.NSET
            self.call_no += 1
            if n:
                self.pool.append_suffix_attention(prms[l], self.sk[c, :n], self.sv[c, :n], self.q[c, :n],
                                                  self.out[c, :n], workspace=self.ws, stream=stream)
        if ev is not None:
            ev[1].record(stream)
        lk = np.array([self.pvalid[r] for r in t.request_ids], np.float64) + TQ
        flop = float((4.0 * TQ * HQ * lk * D).sum()) * N_LAYERS
        b_kv = 34.0 / 32.0
        byts = float((TQ * HQ * D * 2 * 2 + 2 * HKV * (lk - TQ) * D * b_kv + 2 * HKV * TQ * D * 2).sum()) * N_LAYERS
        done = self.sched.end_tick()
        for r in done:
            del self.pvalid[r]
        self.tick_no += 1
        return dict(qtok=n * TQ * N_LAYERS, flop=flop, bytes=byts, reused=t.blocks_reused,
                    admitted=len(t.admitted_index), active=n, completed=len(done))


def run_serve(args, cfg):
    """BASELINE config 5 through the batching scheduler: the same JSON contract, weak scaling (each
    rank serves its own request stream with 256 active), no data-path collective."""
    import torch
    import torch.distributed as dist
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
    free, _ = torch.cuda.mem_get_info(local)
    pool_gb = min(args.pool_gb, free / 1e9 - 12.0)  # room for the inputs and the context
    wl = ServeWorkload(cfg, 1234 + rank, local, pool_gb)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup * N_STEPS):
        wl.tick(stream)
    torch.cuda.synchronize()
    if wl.pool.status() != 0:
        raise RuntimeError("device status word set during warm-up")
    uuid = str(torch.cuda.get_device_properties(local).uuid)
    clocks = Clocks(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    n_ticks = args.steps * N_STEPS
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_ticks)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = wl.ekv.lib.ekv_launch_count()
    tot = dict(qtok=0, flop=0.0, bytes=0.0, reused=0, admitted=0, completed=0, active=0)
    t_start.record(stream)
    for k in range(n_ticks):
        r = wl.tick(stream, evs[k])
        for key in tot:
            tot[key] += r[key]
    t_end.record(stream)
    torch.cuda.synchronize()
    launches = wl.ekv.lib.ekv_launch_count() - n0
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = dispatch.max_over_ranks(t_start.elapsed_time(t_end), device=f"cuda:{local}")
    attn_s = sum(a.elapsed_time(b) for a, b in evs) / 1e3
    n_calls = n_ticks * N_LAYERS
    call_s = attn_s / n_calls
    peaks = load_peaks()
    ach = tot["flop"] / attn_s / 1e12
    roof = {"bound": "tensor", "achieved": ach, "peak": peaks["tc"], "unit": "TFLOP/s", "frac": ach / peaks["tc"],
            "traffic": None, "peak_source": peaks["source"] + " (burst bf16 figure)", "avg_launch_us": call_s * 1e6,
            "kernel": "attn_pair_kernel<Q8>",
            "algorithmic_per_launch": {"flop": tot["flop"] / n_calls, "bytes": tot["bytes"] / n_calls},
            "timed": "CUDA events around each tick's 18 ekv_append_suffix_attention calls, divided by the calls"}
    status = wl.pool.status()
    line = {"metric": METRIC, "value": world * tot["qtok"] / (ms / 1e3), "unit": "query-tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 MMA, f32 accumulate (Q8_0 cache)",
            "data": "synthetic",
            "config": {"workload": args.workload, "description": cfg["desc"], "max_active_per_gpu": wl.B,
                       "pool_gb": round(wl.pool_gb, 1), "pool_blocks": wl.n_blocks,
                       "step": "10 scheduler ticks (one denoise step of every active request each)",
                       "parallelism": f"request-sharded x{world}", "l2": "inputs > L2 (36 distinct call sets)"},
            "serving": {"avg_active": tot["active"] / n_ticks, "admitted_per_step": tot["admitted"] / args.steps,
                        "completed_per_step": tot["completed"] / args.steps,
                        "blocks_reused_per_step": tot["reused"] / args.steps,
                        "timing": "CUDA events from the first to the last tick, host scheduling and prefix "
                                  "appends inside"},
            "roofline": roof, "clocks": clk, "gpu_launches": int(launches), "device_status": status}
    wl.sched.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_other(args, cfg):
    """Configs 3 and 4: the same JSON contract as the default config, without the end-to-end and CPU
    legs (the headline metric is config 2's). Under torchrun every rank runs its own copy of the
    workload -- GR00T: its own 128 requests; LingBot: its own episode (one per GPU) -- with no
    data-path collective; the time is the maximum over ranks."""
    import torch
    import torch.distributed as dist
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
    cls = {"groot": GrootWorkload, "lingbot": LingbotWorkload, "proj": ProjWorkload}[cfg["kind"]]
    wl = cls(cfg["batch"], local)
    stream = torch.cuda.current_stream()
    wl.step_prefix(stream)
    wl.step_calls(stream)
    torch.cuda.synchronize()
    if wl.graphable:
        g_pre, g_calls = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        n0 = wl.ekv.lib.ekv_launch_count()
        with torch.cuda.graph(g_pre, capture_error_mode="thread_local"):
            wl.step_prefix(torch.cuda.current_stream())
        with torch.cuda.graph(g_calls, capture_error_mode="thread_local"):
            wl.step_calls(torch.cuda.current_stream())
        per_step = wl.ekv.lib.ekv_launch_count() - n0
        run_pre, run_calls = g_pre.replay, g_calls.replay
    else:
        run_pre = lambda: wl.step_prefix(torch.cuda.current_stream())
        run_calls = lambda: wl.step_calls(torch.cuda.current_stream())
        per_step = None
    for _ in range(args.warmup):
        run_pre()
        run_calls()
    torch.cuda.synchronize()
    if wl.pool.status() != 0:
        raise RuntimeError("device status word set during warm-up")
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    uuid = str(torch.cuda.get_device_properties(local).uuid)
    clocks = Clocks(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = wl.ekv.lib.ekv_launch_count()
    t_start.record(stream)
    for k in range(args.steps):
        run_pre()
        starts[k].record(stream)
        run_calls()
        ends[k].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    launches = per_step * args.steps if per_step is not None else wl.ekv.lib.ekv_launch_count() - n0
    ms = dispatch.max_over_ranks(t_start.elapsed_time(t_end), device=f"cuda:{local}")
    call_s = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends)) / 1e3 / wl.n_calls
    peaks = load_peaks()
    bound = "tensor" if wl.flop_per_call / (peaks["tc"] * 1e12) >= wl.bytes_per_call / (peaks["hbm"] * 1e9) else "hbm"
    if bound == "tensor":
        ach = wl.flop_per_call / call_s / 1e12
        roof = {"bound": bound, "achieved": ach, "peak": peaks["tc"], "unit": "TFLOP/s", "frac": ach / peaks["tc"]}
    else:
        ach = wl.bytes_per_call / call_s / 1e9
        roof = {"bound": bound, "achieved": ach, "peak": peaks["hbm"], "unit": "GB/s", "frac": ach / peaks["hbm"]}
    roof.update({"traffic": None, "peak_source": peaks["source"], "avg_launch_us": call_s * 1e6,
                 "kernel": {"groot": "attn_heads_kernel (four heads of a request per unit, persistent CTAs)",
                            "lingbot": "attn_tc_kernel (one CTA per 128 query rows)",
                            "proj": "project_qkv_kernel<256> (tcgen05 GEMM, RoPE + slot-write epilogue)"}[cfg["kind"]],
                 "algorithmic_per_launch": {"flop": wl.flop_per_call, "bytes": wl.bytes_per_call},
                 "timed": "CUDA events around each step's layer-calls, divided by the calls (appends included "
                          "for the LingBot chunks)"})
    metric = "denoise qkv-projection tok/s" if cfg["kind"] == "proj" else METRIC
    line = {"metric": metric, "value": world * wl.qtok_per_step * args.steps / (ms / 1e3),
            "unit": "tok/s" if cfg["kind"] == "proj" else "query-tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 MMA, f32 accumulate",
            "data": "synthetic", "config": {"workload": args.config if not args.batch else f"{args.config}@batch{args.batch}",
                                            "description": cfg["desc"],
                                            "batch_per_gpu": wl.B,
                                            "parallelism": f"{'episode' if cfg['kind'] == 'lingbot' else 'request'}"
                                                           f"-sharded x{world}"},
            "roofline": roof, "clocks": clk, "gpu_launches": int(launches), "device_status": wl.pool.status()}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------
# CPU baseline: the oracle (C restatement of the reference's per-call work), all host cores
# ------------------------------------------------------------------------------------------
def cpu_baseline(wl: Pi05Workload, n_req: int, n_layers: int, threads: int):
    """Times the oracle on the first n_req requests x n_layers layer-calls of denoise step 0,
    with the same inputs (copied back from the device)."""
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    import ctypes as C

    B = n_req
    plen = wl.plen[:B]
    maxp = int(plen.max())
    row = HKV * D
    is_q8 = wl.dtype == wl.ekv.DTYPE_Q8_0
    rb = row // 32 * 34 if is_q8 else row * 2
    pk = np.zeros((n_layers, B, maxp, rb), np.uint8)
    pv = np.zeros_like(pk)
    src_row = np.concatenate([[0], np.cumsum(wl.plen)[:-1]])
    for l in range(n_layers):
        for b in range(B):
            n = int(plen[b])
            kb = wl.pk[l, src_row[b]:src_row[b] + n].float().cpu().numpy().reshape(n, row)
            vb = wl.pv[l, src_row[b]:src_row[b] + n].float().cpu().numpy().reshape(n, row)
            if is_q8:
                pk[l, b, :n] = oracle.quantize_q8_0(kb)
                pv[l, b, :n] = oracle.quantize_q8_0(vb)
            else:
                pk[l, b, :n] = oracle.f32_to_bf16(kb).view(np.uint8)
                pv[l, b, :n] = oracle.f32_to_bf16(vb).view(np.uint8)
    sk = wl.sk[:n_layers, :B].contiguous().view(torch.int16).cpu().numpy()
    sv = wl.sv[:n_layers, :B].contiguous().view(torch.int16).cpu().numpy()
    q = wl.q[:n_layers, :B].contiguous().view(torch.int16).cpu().numpy()
    out = np.zeros((B, TQ, HQ, D), np.float32)
    np_ = np.ascontiguousarray(plen, np.int32)
    nv_ = np.ascontiguousarray(wl.pvalid[:B], np.int32)
    args = oracle.CacheArgs(B, TQ, HQ, HKV, D, n_layers, 1 if is_q8 else 0, maxp, TQ, SCALE,
                            np_.ctypes.data, nv_.ctypes.data, pk.ctypes.data, pv.ctypes.data,
                            sk.ctypes.data, sv.ctypes.data, q.ctypes.data, n_layers, out.ctypes.data)
    t0 = time.perf_counter()
    rc = oracle.cache_attention_run(args, threads)
    dt = time.perf_counter() - t0
    assert rc == 0
    qtok = B * TQ * n_layers
    # parity of the timed sample's last call against the GPU output of the same call
    got = wl.out[n_layers - 1, :B].float().cpu().numpy()
    err = float(np.abs(got - out).max())
    return qtok / dt, dt, qtok, err


def pi05_config(args, cfg, world) -> dict:
    """The `config` of a pi0.5 bench line; both arms print the same one."""
    return {"workload": args.workload, "description": cfg["desc"], "batch_per_gpu": cfg["batch"],
            "layers": N_LAYERS, "denoise_steps": N_STEPS, "suffix_tokens": TQ, "q_heads": HQ, "kv_heads": HKV,
            "head_dim": D, "block_tokens": BT, "parallelism": f"request-sharded x{world}",
            "l2": "inputs > L2: every layer-call reads its own Q, suffix K/V and prefix K/V (GBs per step)"}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ------------------------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args, cfg):
    """The reference arm: the reference's CPU path (the oracle port of it; the ggml CPU backend
    it restates is not buildable here) on the host cores, bounded sample per step."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    threads = len(os.sched_getaffinity(0)) or 1
    rng = np.random.default_rng(1234)
    # the sample the GPU arm's cpu_baseline times: 16 requests x the 18 layer-calls of one denoise step
    B = min(cfg["batch"], 16)
    n_layers = N_LAYERS
    reqs = dispatch.make_requests(B, cfg["plo"], cfg["phi"], seed=1234, padded=cfg["padded"])
    plen = np.array([r.prefix_len for r in reqs], np.int32)  # the GPU arm's first B requests
    pvalid = np.array([r.prefix_valid for r in reqs], np.int32)
    maxp = int(plen.max())
    row = HKV * D
    is_q8 = cfg["dtype"] == "q8_0"
    x = (rng.standard_normal((n_layers, B, maxp, row), dtype=np.float32) * 0.5)
    xv = (rng.standard_normal((n_layers, B, maxp, row), dtype=np.float32) * 0.5)
    if is_q8:
        pk = oracle.quantize_q8_0(oracle.bf16_to_f32(oracle.f32_to_bf16(x)))
        pv = oracle.quantize_q8_0(oracle.bf16_to_f32(oracle.f32_to_bf16(xv)))
    else:
        pk = oracle.f32_to_bf16(x).view(np.uint8)
        pv = oracle.f32_to_bf16(xv).view(np.uint8)
    sk = oracle.f32_to_bf16(rng.standard_normal((n_layers, B, TQ, HKV, D), dtype=np.float32) * 0.5)
    sv = oracle.f32_to_bf16(rng.standard_normal((n_layers, B, TQ, HKV, D), dtype=np.float32) * 0.5)
    q = oracle.f32_to_bf16(rng.standard_normal((n_layers, B, TQ, HQ, D), dtype=np.float32) * 0.5)
    out = np.zeros((B, TQ, HQ, D), np.float32)
    args_c = oracle.CacheArgs(B, TQ, HQ, HKV, D, n_layers, 1 if is_q8 else 0, maxp, TQ, SCALE,
                              plen.ctypes.data, pvalid.ctypes.data, pk.ctypes.data, pv.ctypes.data,
                              sk.ctypes.data, sv.ctypes.data, q.ctypes.data, n_layers, out.ctypes.data)
    for _ in range(args.warmup):
        oracle.cache_attention_run(args_c, threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.cache_attention_run(args_c, threads)
        times.append(time.perf_counter() - t0)
    qtok = B * TQ * n_layers
    tot = sum(times)
    value = qtok * len(times) / tot
    sample = f"{B} requests x {n_layers} layer-calls of one denoise step per timed step"
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "query-tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": pi05_config(args, cfg, world),
            "cpu_baseline": {"value": value, "unit": "query-tok/s", "cores": threads, "kind": "port",
                             "sample": sample, "cpu_model": cpu_model()},
            "e2e": {"value": value, "unit": "query-tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ekv", choices=["ekv", "reference"])
    ap.add_argument("--config", default="pi05_q8_b64", choices=sorted(CONFIGS) + sorted(OTHER_CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--batch", type=int, default=0, help="override the requests per GPU (profiling cases)")
    ap.add_argument("--pool-gb", type=float, default=150.0, help="serve_q8_b256: pool size per GPU")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.config in OTHER_CONFIGS:
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"{args.config}: the reference arm times the "
                                  "default pi0.5 workload only"}))
            return
        cfg = dict(OTHER_CONFIGS[args.config])
        if args.batch:
            cfg["batch"] = args.batch  # a profiling case, not the headline config
        run_other(args, cfg)
        return
    cfg = dict(CONFIGS[args.config])
    args.workload = args.config
    if args.batch:
        cfg["batch"] = args.batch
        args.workload = f"{args.config}@batch{args.batch}"  # a profiling case, not the headline config
    if args.impl == "reference":
        run_reference(args, cfg)
        return
    if args.config == "serve_q8_b256":
        run_serve(args, cfg)
        return

    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    # pinned host buffers (the end-to-end leg) local to this GPU's NUMA node
    all_cpus = os.sched_getaffinity(0)
    numa_cpus = dispatch.bind_to_gpu_numa_node(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))

    def barrier():
        if world > 1:
            dist.barrier()

    # rank 0 draws the whole job's request table and scatters each rank its (length-balanced) share
    table = dispatch.make_requests(cfg["batch"] * world, cfg["plo"], cfg["phi"], seed=1234,
                                   padded=cfg["padded"]) if rank == 0 else None
    mine = dispatch.scatter_requests(table, world, rank, "balanced")
    wl = Pi05Workload(cfg, mine, device=local)
    stream = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]

    # One eager step (first-call set-up: kernel attributes, tensor-map encoder), then the step
    # captured as two CUDA graphs -- the 18 prefix appends, and the 180 layer-step calls -- the
    # way the reference runs its denoise loop as one ggml graph. Launches are counted at capture.
    # Thread-local capture: CUDA calls of other threads (the NCCL watchdog under torchrun) do not
    # invalidate it.
    wl.step(stream)
    torch.cuda.synchronize()
    g_pre, g_calls = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    n0 = wl.ekv.lib.ekv_launch_count()
    with torch.cuda.graph(g_pre, capture_error_mode="thread_local"):
        wl.step_prefix(torch.cuda.current_stream())
    with torch.cuda.graph(g_calls, capture_error_mode="thread_local"):
        wl.step_calls(torch.cuda.current_stream())
    launches_per_step = wl.ekv.lib.ekv_launch_count() - n0
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        g_pre.replay()
        g_calls.replay()
    torch.cuda.synchronize()
    if wl.pool.status() != 0:
        raise RuntimeError("device status word set during warm-up")

    uuid = str(torch.cuda.get_device_properties(local).uuid)
    clocks = Clocks(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for k in range(args.steps):
        g_pre.replay()
        starts[k].record(stream)
        g_calls.replay()
        ends[k].record(stream)
    t_end.record(stream)
    launches = launches_per_step * args.steps
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = dispatch.max_over_ranks(t_start.elapsed_time(t_end), device=f"cuda:{local}")
    ms_per_step = ms / args.steps
    value = world * wl.qtok_per_step * args.steps / (ms / 1e3)
    attn_ms = [s.elapsed_time(e) / wl.n_calls for s, e in zip(starts, ends)]  # per layer-step call
    attn_avg_s = statistics.mean(attn_ms) / 1e3
    status = wl.pool.status()

    peaks = load_peaks()
    flop_t = wl.flop_per_call / (peaks["tc"] * 1e12)
    byte_t = wl.bytes_per_call / (peaks["hbm"] * 1e9)
    bound = "tensor" if flop_t >= byte_t else "hbm"
    if bound == "tensor":
        achieved = wl.flop_per_call / attn_avg_s / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peaks["tc"], "unit": "TFLOP/s",
                "frac": achieved / peaks["tc"]}
    else:
        achieved = wl.bytes_per_call / attn_avg_s / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm"], "unit": "GB/s",
                "frac": achieved / peaks["hbm"]}
    roof["traffic"] = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            roof["traffic"] = json.load(f).get(args.workload)
    roof["peak_source"] = peaks["source"] + " (burst bf16 figure)"
    # the library's default tcgen05 kernel at head_dim 256 (EKV_ALGO_TC): CTA pairs
    roof["kernel"] = "attn_pair_kernel<Q8>" if wl.dtype == wl.ekv.DTYPE_Q8_0 else "attn_pair_kernel<bf16>"
    roof["avg_launch_us"] = attn_avg_s * 1e6
    roof["timed"] = ("the 180 ekv_append_suffix_attention calls of each step (one attention launch each at "
                     "head_dim 256, plus the key-split merge where splits are used), CUDA events around "
                     "their graph's replay on the launching stream, divided by 180")
    roof["algorithmic_per_launch"] = {"flop": wl.flop_per_call, "bytes": wl.bytes_per_call}

    # ---- end to end through the C-ABI with host buffers (pinned), copies inside the timing ----
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(wl, args, world, rank, barrier)
        e2e["host_cpus"] = f"{len(numa_cpus)} CPUs of the GPU's NUMA node" if numa_cpus else "unbound"
    os.sched_setaffinity(0, all_cpus)  # the CPU baseline uses the whole host

    line = {"metric": METRIC, "value": value, "unit": "query-tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16/bf16 MMA, f32 accumulate (Q8_0 cache)" if wl.dtype == wl.ekv.DTYPE_Q8_0
            else "bf16 MMA, f32 accumulate",
            "data": "synthetic", "config": pi05_config(args, cfg, world),
            "roofline": roof, "clocks": clk, "gpu_launches": int(launches),
            "device_status": status}
    if e2e is not None:
        line["e2e"] = e2e
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the reference's own thread count, min(hardware threads, 8) (models/pi05.cpp:586-587), and
        # every host thread
        hw = len(all_cpus)
        threads = min(hw, 8)
        v, dt, qtok, err = cpu_baseline(wl, n_req=min(wl.B, 16), n_layers=N_LAYERS, threads=threads)
        v_all, dt_all, _, _ = cpu_baseline(wl, n_req=min(wl.B, 16), n_layers=N_LAYERS, threads=hw)
        line["cpu_baseline"] = {"value": v, "unit": "query-tok/s", "cores": threads, "kind": "port",
                                "sample": f"{min(wl.B, 16)} requests x {N_LAYERS} layer-calls (denoise step 0), "
                                          f"{qtok} query-tokens in {dt:.2f} s",
                                "all_threads": {"value": v_all, "cores": hw, "seconds": dt_all},
                                "cpu_model": cpu_model(), "max_abs_err_vs_gpu": err}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_e2e(wl, args, world, rank, barrier):
    """Same metric through the C-ABI with host buffers: every step copies its inputs from
    pinned host memory (prefix K/V of all layers, per-call suffix K/V and Q) and reads every
    call's output back. Per-call inputs and outputs move in chunks of one denoise step's 18
    layer-calls (one copy per tensor and chunk), double-buffered on separate copy streams so that
    the copies overlap the compute of the neighbouring chunk."""
    import torch
    dev = wl.q.device
    hp = lambda t: torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h_pk, h_pv, h_sk, h_sv, h_q, h_out = hp(wl.pk), hp(wl.pv), hp(wl.sk), hp(wl.sv), hp(wl.q), hp(wl.out)
    h_pk.copy_(wl.pk)
    h_pv.copy_(wl.pv)
    h_sk.copy_(wl.sk)
    h_sv.copy_(wl.sv)
    h_q.copy_(wl.q)
    N, G = wl.n_calls, N_LAYERS
    assert N % G == 0
    # device staging: two chunk slots per per-call tensor
    d_pk, d_pv = torch.empty_like(wl.pk), torch.empty_like(wl.pv)
    slot = lambda t: torch.empty((2, G) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
    d_sk, d_sv, d_q, d_out = slot(wl.sk), slot(wl.sv), slot(wl.q), slot(wl.out)
    s_c = torch.cuda.current_stream()
    s_h2d, s_d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    h2d_bytes = (wl.pk.numel() + wl.pv.numel() + wl.sk.numel() + wl.sv.numel() + wl.q.numel()) * 2
    d2h_bytes = wl.out.numel() * 2
    # the step's result for the serving front: the last layer-step's outputs of every request, gathered
    # on rank 0 over NCCL (the north star's "gather action outputs") and read back there
    h_final = torch.empty((world,) + tuple(wl.out.shape[1:]), dtype=wl.out.dtype, pin_memory=True) if rank == 0 \
        else None
    if rank == 0 and world > 1:
        d2h_bytes += h_final.numel() * 2

    def one_step():
        with torch.cuda.stream(s_h2d):
            d_pk.copy_(h_pk, non_blocking=True)
            d_pv.copy_(h_pv, non_blocking=True)
        pre = torch.cuda.Event()
        pre.record(s_h2d)
        s_c.wait_event(pre)
        for l in range(N_LAYERS):
            wl.pool.append(l, wl.seq_ids, wl.zeros, wl.n_rows, wl.src_row, int(wl.plen.max()), d_pk[l], d_pv[l],
                           stream=s_c)

        def stage(k):  # chunk k = calls [k * G, (k + 1) * G)
            i, cs = k & 1, slice(k * G, (k + 1) * G)
            with torch.cuda.stream(s_h2d):
                s_h2d.wait_event(ev_done[i])  # slot free once chunk k-2 finished reading it
                d_sk[i].copy_(h_sk[cs], non_blocking=True)
                d_sv[i].copy_(h_sv[cs], non_blocking=True)
                d_q[i].copy_(h_q[cs], non_blocking=True)
                ev_in[i].record(s_h2d)

        n_chunks = N // G
        stage(0)
        for k in range(n_chunks):
            i = k & 1
            if k + 1 < n_chunks:
                stage(k + 1)
            s_c.wait_event(ev_in[i])
            s_c.wait_event(ev_out[i])  # output slot drained (chunk k-2)
            for g in range(G):
                l = (k * G + g) % N_LAYERS
                wl.pool.append_suffix_attention(wl.params[l], d_sk[i, g], d_sv[i, g], d_q[i, g], d_out[i, g],
                                                workspace=wl.ws, stream=s_c)
            ev_done[i].record(s_c)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(ev_done[i])
                h_out[k * G:(k + 1) * G].copy_(d_out[i], non_blocking=True)
                ev_out[i].record(s_d2h)
        if world > 1:
            final = dispatch.gather_outputs(d_out[(n_chunks - 1) & 1, G - 1], world, rank)
            if rank == 0:
                h_final.copy_(final, non_blocking=True)

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    torch.cuda.synchronize()
    dt = dispatch.max_over_ranks(time.perf_counter() - t0, device=dev)
    barrier()
    # the host buffers received the same outputs the device-resident run produced
    ok = bool(torch.equal(h_out[-1].to(dev), wl.out[-1]))
    ok_final = True
    if world > 1 and rank == 0:
        ok_final = bool(torch.equal(h_final[0].to(dev), wl.out[-1]))
    return {"value": world * wl.qtok_per_step * args.steps / dt, "unit": "query-tok/s",
            "h2d_bytes_per_step": int(h2d_bytes), "d2h_bytes_per_step": int(d2h_bytes),
            "gather": "NCCL gather of every rank's last layer-step outputs to rank 0, read back there"
                      if world > 1 else None, "gathered_outputs_match": ok_final,
            "ms_per_step": 1e3 * dt / args.steps, "outputs_match_device_run": ok,
            "timing": "host wall clock around K steps, synchronised on both sides"}


if __name__ == "__main__":
    main()
