"""Generate the golden fixtures in tests/golden/ (run once in a container that has gguf-py).

Sources of truth, none of them this repository's own code:
  * gguf-py (installed package `gguf`, quants.py): Q8_0.quantize_blocks / dequantize_blocks and
    BF16.quantize_blocks, whose docstring states bit-exactness with ggml-quants.c. Vectors are
    seeded random data plus hand-picked edge cases (zero blocks, exact .5 ties after scaling,
    fp16-subnormal scales, large magnitudes, NaN/Inf for BF16).
  * numpy's float32 -> float16 conversion (how gguf-py stores the Q8_0 scale).
  * The LingBot CUDA smoke test's known-answer inputs: the formulas, mask and tolerance of
    kernels/lingbot/lingbot_flex_attn_cuda.cu:1033-1076 (S=8, H=2, D=8, causal window 4),
    with its CPU dense reference (:1010-1031) evaluated here in float64.
  * Dense mask matrices built by the loops of the reference mask builders
    (models/smolvla.cpp:705-725, models/hy_vla.cpp:2355-2367, models/groot_n1.cpp:708-718)
    restated over numpy arrays, for small shapes.
  * LingBot-VA flex masks: the token metadata of build_flex_mask_meta and the dense masks of
    flex_self_allowed / flex_cross_allowed (models/lingbot_va.cpp:9283-9348) restated over Python
    lists for three small layouts.
  * Rotary position embedding in the split-halves (NEOX) convention: the installed transformers
    package's Gemma helpers (rotate_half, apply_rotary_pos_emb) in float64, with the frequencies
    1 / base^(2i / head_dim) of its Gemma rotary embedding -- the convention ggml_rope_ext's
    GGML_ROPE_TYPE_NEOX mode implements (models/pi05.cpp:391-401).

Usage:  python tests/golden/make_golden.py      (writes *.npz next to this file)
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def q8_0_vectors():
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as T

    rng = np.random.default_rng(20260101)
    blocks = [rng.standard_normal((48, 32)).astype(np.float32) * 0.5,
              rng.standard_normal((16, 32)).astype(np.float32) * 300.0,
              rng.standard_normal((16, 32)).astype(np.float32) * 1e-6]
    edge = np.zeros((8, 32), np.float32)
    # block 0: all zeros (d = 0, id = 0)
    # block 1: max 127 so id = 1 and x*id lands exactly on .5 ties
    edge[1, :] = np.arange(32, dtype=np.float32) - 16.5
    edge[1, 0] = 127.0
    # block 2: negative max magnitude and ties on the other side
    edge[2, :] = -(np.arange(32, dtype=np.float32) * 0.5 + 0.25)
    edge[2, 5] = -127.0
    # block 3: a single non-zero value
    edge[3, 7] = 3.0e-3
    # block 4: fp16-subnormal scale
    edge[4, :] = np.linspace(-2e-6, 2e-6, 32, dtype=np.float32)
    # block 5: bf16-representable values typical of the N(0,1)*0.5 inputs
    edge[5, :] = np.round(rng.standard_normal(32) * 0.5 * 128) / 128
    # block 6: values whose scaled magnitude is just under / over a half
    edge[6, :] = (np.arange(32, dtype=np.float32) + 0.5) * (1.0 / 127.0) * 4.0
    edge[6, 31] = 1.0
    # block 7: large range
    edge[7, :] = np.geomspace(1e-3, 6e4, 32, dtype=np.float32) * np.where(np.arange(32) % 2, 1, -1)
    x = np.concatenate(blocks + [edge], axis=0).astype(np.float32)
    q = quants.quantize(x, T.Q8_0)
    dq = quants.dequantize(q, T.Q8_0)
    return {"x": x, "q8_0": np.asarray(q, np.uint8), "dequant": np.asarray(dq, np.float32)}


def bf16_vectors():
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as T

    rng = np.random.default_rng(7)
    x = np.concatenate([
        rng.standard_normal(4096).astype(np.float32) * 0.5,
        rng.standard_normal(256).astype(np.float32) * 1e30,
        rng.standard_normal(256).astype(np.float32) * 1e-38,
        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8,
                  1.0 + 2.0 ** -8 + 2.0 ** -20, 3.3895314e38, -3.3895314e38], np.float32),
    ]).astype(np.float32)
    bits = np.asarray(quants.quantize(x.reshape(1, -1), T.BF16), np.uint8).view(np.uint16).ravel()
    return {"x": x, "bf16": bits}


def f16_vectors():
    rng = np.random.default_rng(11)
    x = np.concatenate([
        rng.standard_normal(4096).astype(np.float32),
        rng.standard_normal(512).astype(np.float32) * 1e-5,   # fp16 subnormals
        rng.standard_normal(512).astype(np.float32) * 3e4,
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 70000.0, 2.0 ** -24, 2.0 ** -25,
                  1.5 * 2.0 ** -25, 2.0 ** -26, 6.1035156e-05, 1.0 / 127.0, 127.0 / 127.0],
                 np.float32),
    ]).astype(np.float32)
    return {"x": x, "f16": x.astype(np.float16).view(np.uint16)}


def lingbot_smoke():
    """kernels/lingbot/lingbot_flex_attn_cuda.cu:1034-1047 inputs, dense_ref :1010-1031."""
    S, H, D = 8, 2, 8
    i = np.arange(S * H * D, dtype=np.float32)
    q = (np.sin(i * np.float32(0.017)) * np.float32(0.2)).astype(np.float32)
    k = (np.cos(i * np.float32(0.019)) * np.float32(0.15)).astype(np.float32)
    v = (np.sin(i * np.float32(0.023)) * np.float32(0.3)).astype(np.float32)
    s_idx, t_idx = np.meshgrid(np.arange(S), np.arange(S), indexing="ij")
    mask = ((t_idx <= s_idx) & ((s_idx - t_idx) <= 4)).astype(np.uint8)
    q3 = q.reshape(S, H, D).astype(np.float64)
    k3 = k.reshape(S, H, D).astype(np.float64)
    v3 = v.reshape(S, H, D).astype(np.float64)
    scale = 1.0 / np.sqrt(np.float32(D))
    ref = np.zeros((S, H, D), np.float64)
    for s in range(S):
        for h in range(H):
            allowed = np.nonzero(mask[s])[0]
            dots = (k3[allowed, h, :] @ q3[s, h, :]) * scale
            w = np.exp(dots - dots.max())
            ref[s, h] = (w[:, None] * v3[allowed, h, :]).sum(0) / w.sum()
    return {"q": q.reshape(S, H, D), "k": k.reshape(S, H, D), "v": v.reshape(S, H, D),
            "mask": mask, "ref": ref, "scale": np.float32(scale), "tol": np.float64(1e-5)}


def mask_builders():
    out = {}
    # SmolVLA full mask (models/smolvla.cpp:705-725): n_prefix keys with validity, then a
    # causal suffix of n_suf keys; rows are suffix queries.
    n_prefix, n_suf = 12, 5
    prefix_valid = np.array([1] * 9 + [0] * 3, np.uint8)
    n_total = n_prefix + n_suf
    fm = np.zeros((n_suf, n_total), np.float32)
    for q in range(n_suf):
        for k in range(n_prefix):
            if not prefix_valid[k]:
                fm[q, k] = -np.inf
        for k in range(q + 1, n_suf):
            fm[q, n_prefix + k] = -np.inf
    out["smolvla_full"] = fm
    out["smolvla_meta"] = np.array([n_prefix, 9, n_suf], np.int32)
    # HY-VLA joint mask (models/hy_vla.cpp:2355-2367): prefix visible, suffix row 0 sees only
    # suffix key 0.
    n_pref, n_suf2 = 10, 6
    full = np.zeros((n_suf2, n_pref + n_suf2), np.float32)
    for r in range(n_suf2):
        for c in range(n_pref + n_suf2):
            allowed = c < n_pref
            if not allowed:
                s = c - n_pref
                allowed = (s == 0) if r == 0 else True
            full[r, c] = 0.0 if allowed else -np.inf
    out["hyvla_full"] = full
    out["hyvla_meta"] = np.array([n_pref, n_suf2], np.int32)
    # GR00T text / image masks (models/groot_n1.cpp:708-718) over a 20-token backbone where
    # tokens 4..13 are image tokens and tokens >= 17 are invalid.
    bb, seq = 20, 3
    valid = np.array([1] * 17 + [0] * 3, np.uint8)
    is_image = np.array([0] * 4 + [1] * 10 + [0] * 6, np.uint8)
    text = np.zeros((seq, bb), np.float32)
    image = np.zeros((seq, bb), np.float32)
    for qq in range(seq):
        for kk in range(bb):
            text[qq, kk] = 0.0 if (valid[kk] and not is_image[kk]) else -np.inf
            image[qq, kk] = 0.0 if (valid[kk] and is_image[kk]) else -np.inf
    out["groot_text"] = text
    out["groot_image"] = image
    out["groot_meta"] = np.array([bb, 17, 4, 14, seq], np.int32)
    return out


def lingbot_flex():
    """LingBot-VA flex masks over the token metadata of build_flex_mask_meta
    (models/lingbot_va.cpp:9283-9334), restated over Python lists: latent tokens (one per
    (frame / pt, h / ph, w / pw) patch, frame id (f * pt) / chunk_size * 2) then action tokens
    (frame id f / chunk_size * 2 + 1), each group first with noise id 0 and then repeated with noise id
    1, then `padded_length` padding tokens (ids -1); text_seq_ids: `text_seq` ids per batch element.
    Dense masks from flex_self_allowed (:9336-9344) and flex_cross_allowed (:9346-9348), for three
    small layouts (one is the runtime layout of build_runtime_flex_meta, :9435-9440, with a
    2-patch latent and a 2-frame action, chunk 1, window 4)."""
    def meta(latent, action, padded_length, chunk_size, window_size, pt, ph, pw, text_seq):
        lb, _, lf, lh, lw = latent
        _, _, af, ah, aw = action
        lat_seq, lat_frame, act_seq, act_frame = [], [], [], []
        for b in range(lb):
            for f in range(lf // pt):
                for h in range(lh // ph):
                    for w in range(lw // pw):
                        lat_seq.append(b)
                        lat_frame.append((f * pt) // chunk_size * 2)
            for f in range(af):
                for h in range(ah):
                    for w in range(aw):
                        act_seq.append(b)
                        act_frame.append(f // chunk_size * 2 + 1)
        seq = lat_seq + lat_seq + act_seq + act_seq + [-1] * padded_length
        frame = lat_frame + lat_frame + act_frame + act_frame + [-1] * padded_length
        noise = [0] * len(lat_seq) + [1] * len(lat_seq) + [0] * len(act_seq) + [1] * len(act_seq) + [-1] * padded_length
        text = [b for b in range(lb) for _ in range(text_seq)]
        n = len(seq)
        self_m = np.zeros((n, n), bool)
        for q in range(n):
            for k in range(n):
                if seq[q] < 0 or seq[q] != seq[k]:
                    continue
                qf, kf, qn, kn = frame[q], frame[k], noise[q], noise[k]
                c2c = qn == 1 and kn == 1 and kf <= qf
                n2c = qn == 0 and kn == 1 and kf < qf
                n2n = qn == 0 and kn == 0 and kf == qf
                self_m[q, k] = (c2c or n2c or n2n) and abs(qf - kf) <= window_size
        cross_m = np.zeros((n, len(text)), bool)
        for q in range(n):
            for k in range(len(text)):
                cross_m[q, k] = seq[q] >= 0 and seq[q] == text[k]
        return (np.array(seq, np.int64), np.array(frame, np.int64), np.array(noise, np.int64),
                np.array(text, np.int64), self_m, cross_m)

    layouts = {
        # (latent b, c, f, h, w), (action b, c, f, h, w), padded, chunk, window, pt, ph, pw, text
        "runtime": ((1, 4, 2, 4, 4), (1, 7, 2, 2, 1), 3, 1, 4, 1, 2, 2, 6),
        "chunks": ((1, 4, 8, 2, 2), (1, 7, 8, 1, 1), 5, 2, 2, 1, 1, 1, 4),
        "batch2": ((2, 4, 4, 2, 2), (2, 7, 4, 1, 1), 2, 1, 1, 1, 2, 1, 3),
    }
    out = {}
    for name, args in layouts.items():
        seq, frame, noise, text, self_m, cross_m = meta(*args)
        out[f"{name}_seq"], out[f"{name}_frame"], out[f"{name}_noise"], out[f"{name}_text"] = seq, frame, noise, text
        out[f"{name}_self"], out[f"{name}_cross"] = self_m, cross_m
        out[f"{name}_window"] = np.array(args[4], np.int64)
    return out


def rope_neox():
    import torch
    from transformers.models.gemma.modeling_gemma import apply_rotary_pos_emb

    rng = np.random.default_rng(20260303)
    base, d = 10000.0, 32
    pos = np.array([0, 1, 7, 50, 816, 865], np.int64)
    x = rng.standard_normal((len(pos), 3, d)).astype(np.float32)
    inv_freq = 1.0 / (base ** (np.arange(0, d, 2, dtype=np.float64) / d))
    ang = pos[:, None].astype(np.float64) * inv_freq[None, :]
    emb = np.concatenate([ang, ang], axis=-1)
    cos, sin = torch.tensor(np.cos(emb)), torch.tensor(np.sin(emb))  # [rows, d]
    xt = torch.tensor(x.astype(np.float64))                            # [rows, heads, d]
    out, _ = apply_rotary_pos_emb(xt, xt, cos, sin, unsqueeze_dim=1)
    return dict(x=x, pos=pos.astype(np.int32), base=np.float64(base), out=out.numpy())


def main():
    np.savez_compressed(os.path.join(HERE, "q8_0_gguf.npz"), **q8_0_vectors())
    np.savez_compressed(os.path.join(HERE, "bf16_gguf.npz"), **bf16_vectors())
    np.savez_compressed(os.path.join(HERE, "f16_numpy.npz"), **f16_vectors())
    np.savez_compressed(os.path.join(HERE, "lingbot_smoke.npz"), **lingbot_smoke())
    np.savez_compressed(os.path.join(HERE, "mask_builders.npz"), **mask_builders())
    np.savez_compressed(os.path.join(HERE, "lingbot_flex.npz"), **lingbot_flex())
    np.savez_compressed(os.path.join(HERE, "rope_neox.npz"), **rope_neox())
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
