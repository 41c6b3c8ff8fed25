#!/usr/bin/env python3
"""Generate tests/golden/gpt2_model_t{T}.npz from the reference's own NumPy
mirror of the fixed-point GPT-2 model (scripts/gpt2_fixed.py forward_model,
stated bit-exact with rust/volta-gpt2's forward).

Run once in a checkout that has the reference tree:
    python tests/golden/make_model_golden.py /path/to/reference [T ...]
    python tests/golden/make_model_golden.py --scaled /path/to/reference [T ...]

--scaled writes gpt2_scaled_t{T}.npz instead: the first 2 layers of the
scaled synthetic shape (24 layers, d_model 1024, 16 heads of 64, MLP 4096),
from the same mirror with its shape constants (D, H, DFF) set to that shape
(every mirror function reads them at call time), every wire of both layers.

The model is the reference's synthetic GPT-2 small
(rust/volta-gpt2/src/model.rs:504-600 synthetic_model, seed 0x1234 as in its
runtime_model test at model.rs:930):
  * layer l's weights = synthetic_weights(seed + l * 0x9E3779B9) (the mirror's
    own splitmix64 generator, layer.rs:283-309), zero GEMM biases;
  * wte (vocab x d, radius 15) then wpe (1024 x d, radius 7) from one LCG
    state seed ^ 0xD1B54A32D192ED03, x <- x * 6364136223846793005 +
    1442695040888963407, value = x mod (2r+1) - r; tied output;
  * final LN gain 64, bias 0; LutParams defaults with the P5 stable softmax
    (softmax_row_shift = true, luts.rs:57-59), shift_embed 0, no seams.  With
    softmax_row_shift = false (LutParams::default) the reference itself
    stops at T = 1024: the softmax reciprocal index leaves its u16 domain
    (layer.rs:782 assert; the mirror raises SaturationError), so the
    T = 1024 prefill needs the row-shifted softmax and its 18-bit
    reciprocal domain.
Tokens: FpStream::domain_separated([0x70; 32], 0).next_fp() mod 50257 (the
oracle's pinned ChaCha8 FpStream).

The fixture holds SHA-256 digests (not tensors): embed_out, every layer's
attn_block_out and ffn_block_out, every intermediate of layers 0 and L-1,
the final LN row and the logits, plus the mirror's saturation stats.
"""

import hashlib
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

SEED = 0x1234
TOKEN_SEED = bytes([0x70] * 32)
VOCAB, POS = 50257, 1024
LAYER_KEYS = ["row_shift", "ln1_out", "qkv_acc", "q", "k", "v", "scores_acc", "scores_q", "exp_out", "denoms", "recips", "av_acc",
              "av_q", "proj_acc", "attn_proj_q", "attn_block_out", "ln2_out", "ffn_up_acc", "ffn_up_q", "gelu_out",
              "ffn_down_acc", "ffn_down_q", "ffn_block_out"]


def digest(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def lcg_values(state: int, n: int, radius: int):
    """n successive LCG draws mapped to [-radius, radius]; returns the values
    and the state after the last draw (pure Python ints, exact)."""
    a, c, m = 6364136223846793005, 1442695040888963407, (1 << 64) - 1
    out = np.empty(n, dtype=np.int16)
    span = 2 * radius + 1
    for i in range(n):
        state = (state * a + c) & m
        out[i] = state % span - radius
    return out, state


def main(ref_root: str, ts, scaled: bool = False):
    sys.path.insert(0, os.path.join(ref_root, "scripts"))
    import gpt2_fixed as g

    from oracle import oracle as o

    D, L = 768, 12
    if scaled:
        D, L = 1024, 2
        g.D, g.H, g.DFF = D, D // g.DH, 4096

    t0 = time.time()
    layers = []
    for layer in range(L):
        w = g.synthetic_weights((SEED + layer * 0x9E3779B9) & 0xFFFFFFFFFFFFFFFF)
        layers.append(dict(c_attn=w.c_attn, attn_proj=w.attn_proj, ffn_up=w.ffn_up, ffn_down=w.ffn_down,
                           ln1_gain=w.ln1_gain, ln1_bias=w.ln1_bias, ln2_gain=w.ln2_gain, ln2_bias=w.ln2_bias))
    state = SEED ^ 0xD1B54A32D192ED03
    wte, state = lcg_values(state, VOCAB * D, 15)
    wpe, state = lcg_values(state, POS * D, 7)
    model = {"layers": layers, "wte": wte.reshape(VOCAB, D), "wpe": wpe.reshape(POS, D),
             "lnf_gain": np.full(D, 64, dtype=np.int16), "lnf_bias": np.zeros(D, dtype=np.int16)}
    print(f"model built in {time.time() - t0:.0f}s", flush=True)
    lp = g.LutParams()
    luts = g.build_luts_p4(lp)
    p = {k: getattr(lp, k) for k in lp.__dataclass_fields__}
    p.update(shift_embed=0, softmax_row_shift=True)
    wdig = digest(np.concatenate([np.concatenate([lw[k].ravel() for k in ("c_attn", "attn_proj", "ffn_up", "ffn_down",
                                                                            "ln1_gain", "ln1_bias", "ln2_gain",
                                                                            "ln2_bias")]) for lw in layers]))
    for t in ts:
        tokens = (o.chacha_fp_rows(TOKEN_SEED, 0, 1, t)[0] % np.uint64(VOCAB)).astype(np.int64)
        t1 = time.time()
        try:
            res = g.forward_model(tokens, model, luts, p, mode="strict")
            strict_ok = True
        except g.SaturationError as e:
            print("strict mode saturated:", e, flush=True)
            res = g.forward_model(tokens, model, luts, p, mode="stats")
            strict_ok = False
        print(f"T={t}: forward in {time.time() - t1:.0f}s, strict={strict_ok}", flush=True)
        out = {"t": np.array(t), "seed": np.array(SEED), "strict_ok": np.array(strict_ok),
               "softmax_row_shift": np.array(True),
               "tokens_digest": np.array(digest(tokens.astype(np.uint32))), "weights_digest": np.array(wdig),
               "wte_digest": np.array(digest(model["wte"])), "wpe_digest": np.array(digest(model["wpe"])),
               "embed_out": np.array(digest(res["embed_out"])), "final_ln_out": np.array(digest(res["final_ln_out"])),
               "logits": np.array(digest(res["logits"])),
               "stats": np.array(json.dumps(res.get("stats", {}), sort_keys=True, default=str))}
        for layer, lr in enumerate(res["layers"]):
            out[f"l{layer}_attn_block_out"] = np.array(digest(lr["attn_block_out"]))
            out[f"l{layer}_ffn_block_out"] = np.array(digest(lr["ffn_block_out"]))
            if layer in (0, L - 1):
                for k in LAYER_KEYS:
                    out[f"l{layer}_{k}"] = np.array(digest(lr[k]))
        name = f"gpt2_scaled_t{t}.npz" if scaled else f"gpt2_model_t{t}.npz"
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), name)
        np.savez_compressed(path, **out)
        print("wrote", path, os.path.getsize(path), "bytes", flush=True)


if __name__ == "__main__":
    argv = sys.argv[1:]
    scaled = bool(argv) and argv[0] == "--scaled"
    argv = argv[1:] if scaled else argv
    if not argv:
        sys.exit("usage: make_model_golden.py [--scaled] <reference checkout> [T ...]")
    main(argv[0], [int(x) for x in argv[1:]] or ([16] if scaled else [16, 1024]), scaled)
