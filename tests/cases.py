"""Shared builders for the GPU parity tests: seeded bf16 inputs, a pool filled through the
C-ABI, and the matching oracle inputs (logical prefix+suffix K/V per request)."""
from __future__ import annotations

import numpy as np
import torch

import ekv
import oracle


def bf16_randn(gen, shape, scale=0.5):
    """N(0,1)*scale rounded to bf16 (RNE), as the BASELINE configs draw Q/K/V."""
    return (torch.randn(shape, generator=gen, dtype=torch.float32) * scale).to(torch.bfloat16)


def to_f32_np(t):
    return t.float().cpu().numpy()


def shuffled_tables(rng, n_blocks_total, need):
    """Disjoint random block lists (a seeded permutation of the pool's blocks)."""
    perm = rng.permutation(n_blocks_total)
    out, o = [], 0
    for n in need:
        out.append([int(x) for x in perm[o:o + n]])
        o += n
    return out


class Filled:
    """A pool with B sequences whose prefix (per layer) and suffix slot are filled."""

    def __init__(self, *, dtype, B, prefix_lens, Hkv, D, n_layers=1, block_tokens=16,
                 suffix_len=0, suffix_cap=None, seed=0, shuffle=True, device="cuda"):
        self.B, self.Hkv, self.D, self.n_layers = B, Hkv, D, n_layers
        self.dtype = dtype
        self.prefix_lens = list(prefix_lens)
        self.suffix_len = suffix_len
        cap = suffix_cap if suffix_cap is not None else suffix_len
        bt = block_tokens
        need = [(n + bt - 1) // bt for n in self.prefix_lens]
        n_blocks = sum(need) + 8
        self.pool = ekv.Pool(device=0, dtype=dtype, block_tokens=bt, n_blocks=n_blocks, kv_heads=Hkv,
                             head_dim=D, n_layers=n_layers, max_seqs=B + 2,
                             max_blocks_per_seq=max(need) + 2, suffix_tokens=cap)
        rng = np.random.default_rng(seed)
        gen = torch.Generator().manual_seed(seed)
        self.seqs = [self.pool.seq_create() for _ in range(B)]
        if shuffle:
            tables = shuffled_tables(rng, n_blocks, need)
            for s, tb, n in zip(self.seqs, tables, self.prefix_lens):
                self.pool.seq_set_blocks(s, tb, n)
        else:
            for s, n in zip(self.seqs, self.prefix_lens):
                self.pool.seq_resize(s, n)
        self.pool.sync()
        self.seq_ids = torch.tensor(self.seqs, dtype=torch.int32, device=device)
        Lmax = max(self.prefix_lens)
        # per layer: prefix K/V [B][Lmax][Hkv][D] bf16 (rows beyond a request's length unused)
        self.pk = [bf16_randn(gen, (B, Lmax, Hkv, D)) for _ in range(n_layers)]
        self.pv = [bf16_randn(gen, (B, Lmax, Hkv, D)) for _ in range(n_layers)]
        self.sk = [bf16_randn(gen, (B, max(suffix_len, 1), Hkv, D)) for _ in range(n_layers)]
        self.sv = [bf16_randn(gen, (B, max(suffix_len, 1), Hkv, D)) for _ in range(n_layers)]
        for l in range(n_layers):
            # ragged append: packed rows, one batch element per request
            rows = [self.pk[l][b, :self.prefix_lens[b]] for b in range(B)]
            rows_v = [self.pv[l][b, :self.prefix_lens[b]] for b in range(B)]
            k_packed = torch.cat(rows).contiguous().to(device)
            v_packed = torch.cat(rows_v).contiguous().to(device)
            src_row = np.concatenate([[0], np.cumsum(self.prefix_lens)[:-1]]).astype(np.int32)
            self.pool.append(l, self.seq_ids,
                             torch.zeros(B, dtype=torch.int32, device=device),
                             torch.tensor(self.prefix_lens, dtype=torch.int32, device=device),
                             torch.tensor(src_row, device=device), Lmax, k_packed, v_packed)
            if suffix_len:
                self.pool.append_suffix(l, self.seq_ids, self.sk[l][:, :suffix_len].contiguous().to(device),
                                        self.sv[l][:, :suffix_len].contiguous().to(device))
        torch.cuda.synchronize()

    def oracle_kv(self, layer):
        """Logical K/V per request as the oracle sees them: [B][Lmax+Ls][Hkv][D] f32."""
        B, Hkv, D = self.B, self.Hkv, self.D
        Lmax = max(self.prefix_lens)
        Ls = self.suffix_len
        k = np.zeros((B, Lmax + Ls, Hkv, D), np.float32)
        v = np.zeros_like(k)
        for b in range(B):
            n = self.prefix_lens[b]
            pk = to_f32_np(self.pk[layer][b, :n])
            pv = to_f32_np(self.pv[layer][b, :n])
            if self.dtype == ekv.DTYPE_Q8_0:
                pk = oracle.dequantize_q8_0(oracle.quantize_q8_0(pk.reshape(n, -1))).reshape(pk.shape)
                pv = oracle.dequantize_q8_0(oracle.quantize_q8_0(pv.reshape(n, -1))).reshape(pv.shape)
            k[b, :n] = pk
            v[b, :n] = pv
            if Ls:
                k[b, n:n + Ls] = to_f32_np(self.sk[layer][b, :Ls])
                v[b, n:n + Ls] = to_f32_np(self.sv[layer][b, :Ls])
        return k, v

    def oracle_kv_compact(self, layer):
        """Per-request key arrays with the suffix directly after each request's own prefix."""
        k, v = self.oracle_kv(layer)
        return k, v
