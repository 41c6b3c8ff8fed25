"""Oracle (test infrastructure only) for the GPT-2 small prefill path.

Whole-model forward: forward_layer / forward_model compose the oracle's
fixed-point primitives (oracle/fixed.c) in the order of the reference's NumPy
mirror scripts/gpt2_fixed.py:427-645 (forward_layer) and 688-760
(forward_model); OracleOps binds them.

Prefill proof schedule: Schedule / pcs_root compose the oracle's restated
primitives into the checker of libvolta_accel.so's Gpt2Prover
(volta_zk_b200/host/gpt2_proof.cpp): LogUp over Fp columns
(logup.rs:1760-1771), the clear product and triple-product sumchecks
(sumcheck_clear.rs:23-70, hadamard.rs:222-240), matrix folds and eq tables
(mle.rs:7-30), ChaCha8 VOLE-MAC masks (corr.rs:234-255) and the Ligero
commitment (ligero.rs:465-505, ntt.rs, merkle.rs); the lookup columns restate
block_proof.rs range_cols_padded / range_mult / pair_cols_padded / pair_table
(2359-2520) in numpy.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs only, as the checker; the shipped library never imports it.
"""

import numpy as np

# GPT-2 small.  Every function below takes its dimensions from the weights
# it is given (d = ln1_gain's length, dff = ffn_up's size / d, heads =
# d / 64; flat arrays work), so the same code checks other shapes such as
# the 24-layer d-1024 one.
D, H, DH, DFF = 768, 12, 64, 3072
# P4 LutParams defaults (gpt2_fixed.py LutParams / luts.rs)
LN_VAR_SHIFT, SHIFT_LN_NORM, RECIP_DEN_SHIFT, RECIP_LOG2 = 7, 16, 6, 26
SHIFT_QKV, SHIFT_SCORES, SHIFT_SOFTMAX_NORM, SHIFT_AV = 10, 10, 14, 12
SHIFT_ATTN_PROJ, SHIFT_FFN_UP, SHIFT_FFN_DOWN = 10, 10, 10


def forward_layer(ops, x, w, luts, t, row_shift=0):
    """forward_layer from the seam primitives; `ops` provides layer_norm,
    gemm, qkv_split, scores, softmax, av, lookup with the oracle's
    signatures.  row_shift = 1 selects the P5 stable softmax.  Returns
    {name: array} with the reference's names."""
    D = np.asarray(w["ln1_gain"]).size
    DFF, H = np.asarray(w["ffn_up"]).size // D, D // DH
    r = {"x_in": x}
    ln1 = ops.layer_norm(x, w["ln1_gain"], w["ln1_bias"], luts["ln_rsqrt"], t, D, LN_VAR_SHIFT, SHIFT_LN_NORM)
    r.update(ln1_mean=ln1[0], ln1_var=ln1[1], ln1_rsqrt_in=ln1[2], ln1_rsqrt_out=ln1[3], ln1_acc=ln1[4],
             ln1_out=ln1[5])
    errs = [ln1[6]]
    qkv_acc, qkv_q, _, e = ops.gemm(ln1[5], w["c_attn"], None, None, t, D, 3 * D, SHIFT_QKV)
    errs.append(e)
    r.update(qkv_acc=qkv_acc, qkv_q=qkv_q)
    q, k, v = ops.qkv_split(qkv_q, t, D)
    r.update(q=q, k=k, v=v)
    s_acc, s_q, e = ops.scores(q, k, t, t, 0, H, DH, SHIFT_SCORES)
    errs.append(e)
    r.update(scores_acc=s_acc, scores_q=s_q)
    rs, exp_out, denoms, recips, wts, e = ops.softmax(s_q, luts["exp"], luts["softmax_recip"], t, 0, H,
                                                      RECIP_DEN_SHIFT, RECIP_LOG2, SHIFT_SOFTMAX_NORM, row_shift)
    errs.append(e)
    r.update(row_shift=rs, exp_out=exp_out, denoms=denoms, recips=recips, weights=wts)
    av_acc, av_q, e = ops.av(wts, v, t, t, 0, D, H, SHIFT_AV)
    errs.append(e)
    r.update(av_acc=av_acc, av_q=av_q)
    proj_acc, proj_q, attn_out, e = ops.gemm(av_q, w["attn_proj"], None, x.reshape(-1), t, D, D, SHIFT_ATTN_PROJ)
    errs.append(e)
    r.update(proj_acc=proj_acc, attn_proj_q=proj_q, attn_block_out=attn_out)
    ln2 = ops.layer_norm(attn_out, w["ln2_gain"], w["ln2_bias"], luts["ln_rsqrt"], t, D, LN_VAR_SHIFT, SHIFT_LN_NORM)
    errs.append(ln2[6])
    r.update(ln2_mean=ln2[0], ln2_var=ln2[1], ln2_rsqrt_in=ln2[2], ln2_rsqrt_out=ln2[3], ln2_acc=ln2[4],
             ln2_out=ln2[5])
    up_acc, up_q, _, e = ops.gemm(ln2[5], w["ffn_up"], None, None, t, D, DFF, SHIFT_FFN_UP)
    errs.append(e)
    r.update(ffn_up_acc=up_acc, ffn_up_q=up_q)
    gelu = ops.lookup(up_q, luts["gelu"])
    r["gelu_out"] = gelu
    dn_acc, dn_q, out, e = ops.gemm(gelu, w["ffn_down"], None, attn_out, t, DFF, D, SHIFT_FFN_DOWN)
    errs.append(e)
    r.update(ffn_down_acc=dn_acc, ffn_down_q=dn_q, ffn_block_out=out)
    r["errors"] = errs
    return r


def forward_model(ops, tokens, model, luts, row_shift=1):
    """gpt2_fixed.py forward_model (688-760) from the same primitives: embed
    (shift 0), every layer, final LN of the last row, its logits against the
    tied wte.  `model` is a volta_zk_b200.gpt2.Gpt2Model."""
    t = len(tokens)
    vocab, D = model.wte.shape
    acc, x, e = ops.embed(tokens, model.wte, model.wpe, t, D, vocab, model.wpe.shape[0], 0, 0)
    out = {"embed_out": x, "errors": [e], "layers": []}
    for lw in model.layers:
        r = forward_layer(ops, x, lw, luts, t, row_shift)
        out["layers"].append(r)
        out["errors"] += r["errors"]
        x = r["ffn_block_out"]
    fin = ops.layer_norm(np.ascontiguousarray(x[-D:]), model.lnf_gain, model.lnf_bias, luts["ln_rsqrt"], 1, D,
                         LN_VAR_SHIFT, SHIFT_LN_NORM)
    out["errors"].append(fin[6])
    out["final_ln_out"] = fin[5]
    out["logits"] = ops.logits(fin[5], model.wte, 1, D, vocab)
    return out


def _tri(x):
    return x * (x + 1) // 2


def band_witness(ops, full, model, luts, t0):
    """band_model_witness (rust/volta-gpt2/src/band.rs:77-196) from a
    forward_model result over t rows: row-local wires sliced to rows t0 .. t-1,
    the per-head causal-packed wires repacked to the band (head h keeps rows
    t0 .. t-1 with their windows t0 + i + 1), the per-head row tables cut to
    h x q, the final LayerNorm over every band row of the last layer's output
    and the logits of every band row."""
    vocab, D = model.wte.shape
    H = D // DH
    t = np.asarray(full["embed_out"]).size // D
    q = t - t0

    def rows(a):
        a = np.asarray(a).reshape(-1)
        width = a.size // t
        return a[t0 * width:t * width]

    layers = []
    for r in full["layers"]:
        b = {}
        for name, v in r.items():
            if name == "errors":
                continue
            if name in ("scores_acc", "scores_q", "exp_out", "weights"):
                b[name] = np.asarray(v).reshape(H, _tri(t))[:, _tri(t0):].reshape(-1)
            elif name in ("row_shift", "denoms", "recips"):
                b[name] = np.asarray(v).reshape(H, t)[:, t0:].reshape(-1)
            else:
                b[name] = rows(v)
        layers.append(b)
    x_fin = np.ascontiguousarray(rows(full["layers"][-1]["ffn_block_out"]))
    fin = ops.layer_norm(x_fin, model.lnf_gain, model.lnf_bias, luts["ln_rsqrt"], q, D, LN_VAR_SHIFT, SHIFT_LN_NORM)
    logits = ops.logits(fin[5], model.wte, q, D, vocab)
    return {"layers": layers, "fin": fin[:6], "fin_error": fin[6], "logits": np.asarray(logits).reshape(q, vocab),
            "embed_out": rows(full["embed_out"])}


def argmax_last(x):
    """decode.rs:270-272: Iterator::max_by_key returns the last of equal maxima."""
    x = np.asarray(x)
    return int(x.size - 1 - int(np.argmax(x[::-1])))


def decode_step(ops, model, luts, cache, token, pos, row_shift=1):
    """decode_step (rust/volta-gpt2/src/decode.rs:137-268) on the oracle's
    primitives: one new row at position pos; its K/V rows are appended to
    `cache` ({"k": [per layer], "v": [per layer]}, pos rows each) before the
    attention over rows 0 .. pos.  Returns (logits row, error flags)."""
    vocab, D = model.wte.shape
    H, DFF = D // DH, np.asarray(model.layers[0]["ffn_up"]).size // D
    _, x, e = ops.embed(np.array([token], np.uint32), model.wte, model.wpe, 1, D, vocab, model.wpe.shape[0], pos, 0)
    errs = [e]
    for l, lw in enumerate(model.layers):
        ln1 = ops.layer_norm(x, lw["ln1_gain"], lw["ln1_bias"], luts["ln_rsqrt"], 1, D, LN_VAR_SHIFT, SHIFT_LN_NORM)
        _, qkv_q, _, e1 = ops.gemm(ln1[5], lw["c_attn"], None, None, 1, D, 3 * D, SHIFT_QKV)
        q, k, v = ops.qkv_split(qkv_q, 1, D)
        cache["k"][l] = np.concatenate([cache["k"][l], k])
        cache["v"][l] = np.concatenate([cache["v"][l], v])
        _, s_q, e2 = ops.scores(q, cache["k"][l], 1, pos + 1, pos, H, DH, SHIFT_SCORES)
        _, _, _, _, wts, e3 = ops.softmax(s_q, luts["exp"], luts["softmax_recip"], 1, pos, H, RECIP_DEN_SHIFT,
                                          RECIP_LOG2, SHIFT_SOFTMAX_NORM, row_shift)
        _, av_q, e4 = ops.av(wts, cache["v"][l], 1, pos + 1, pos, D, H, SHIFT_AV)
        _, _, attn_out, e5 = ops.gemm(av_q, lw["attn_proj"], None, x, 1, D, D, SHIFT_ATTN_PROJ)
        ln2 = ops.layer_norm(attn_out, lw["ln2_gain"], lw["ln2_bias"], luts["ln_rsqrt"], 1, D, LN_VAR_SHIFT,
                             SHIFT_LN_NORM)
        _, up_q, _, e6 = ops.gemm(ln2[5], lw["ffn_up"], None, None, 1, D, DFF, SHIFT_FFN_UP)
        gelu = ops.lookup(up_q, luts["gelu"])
        _, _, x, e7 = ops.gemm(gelu, lw["ffn_down"], None, attn_out, 1, DFF, D, SHIFT_FFN_DOWN)
        errs += [ln1[6], e1, e2, e3, e4, e5, ln2[6], e6, e7]
    fin = ops.layer_norm(x, model.lnf_gain, model.lnf_bias, luts["ln_rsqrt"], 1, D, LN_VAR_SHIFT, SHIFT_LN_NORM)
    errs.append(fin[6])
    return np.asarray(ops.logits(fin[5], model.wte, 1, D, vocab)).reshape(-1), errs


def generate(ops, model, luts, k_rows, v_rows, t0, logits_t0, n, row_shift=1):
    """generate (decode.rs:278-300): greedy steps after a prefill of t0 rows
    whose per-layer K/V (t0 x D) and last-position logits are given.  Returns
    (tokens, logits rows, cache)."""
    D = model.wte.shape[1]
    cache = {"k": [np.asarray(k).reshape(-1)[:t0 * D].copy() for k in k_rows],
             "v": [np.asarray(v).reshape(-1)[:t0 * D].copy() for v in v_rows]}
    tokens, rows, errs = [], [], []
    nxt = argmax_last(logits_t0)
    for i in range(n):
        tokens.append(nxt)
        lg, e = decode_step(ops, model, luts, cache, nxt, t0 + i, row_shift)
        rows.append(lg)
        errs += e
        nxt = argmax_last(lg)
    return tokens, np.stack(rows), cache, errs


class OracleOps:
    def __init__(self, o):
        self.o = o

    def layer_norm(self, *a):
        return self.o.fixed_layer_norm(*a)

    def gemm(self, *a):
        return self.o.fixed_gemm(*a)

    def qkv_split(self, *a):
        return self.o.fixed_qkv_split(*a)

    def scores(self, *a):
        return self.o.fixed_attention_scores(*a)

    def softmax(self, *a):
        return self.o.fixed_softmax(*a)

    def av(self, *a):
        return self.o.fixed_av(*a)

    def lookup(self, x, lut):
        return self.o.fixed_lookup(x, lut)

    def embed(self, tokens, wte, wpe, rows, d, vocab, positions, pos0, shift):
        return self.o.fixed_embed(tokens, wte, wpe, rows, d, vocab, positions, pos0, shift)

    def logits(self, x, w, rows, d, vocab):
        return self.o.fixed_logits(x, w, rows, d, vocab)



P = 0xFFFFFFFF00000001
HEAD_PAD = 16
RECIP_BITS = 18
RECIP_PAD_INPUT = 256
PCS_ROWS, PCS_COL_BITS, PCS_PAD, PCS_CODE_BITS = 8192, 14, 512, 15
SITES = dict(down_range=1, gelu=2, up_range=3, ln2_norm=4, ln2_rsqrt=5, proj_range=6, av_range=7, norm_range=8,
             exp=9, recip=10, scores_range=11, qkv_range=12, ln1_norm=13, ln1_rsqrt=14, gemm_down=16, gemm_up=17,
             ln2_had=18, gemm_proj=19, av=20, norm_had=21, qk=22, gemm_qkv=23, ln1_had=24)


def site_domain(layer, site, chunk=0):
    """Transcript domain of a sub-proof site; chunk 0 is the prefill, c >= 1
    the c-th decode band of a response."""
    return 0x7000000000000000 | (chunk << 32) | (layer << 16) | (SITES[site] << 8)


def pow2(n):
    p = 1
    while p < n:
        p <<= 1
    return p


def emb(v):
    v = np.asarray(v).astype(np.int64)
    return np.where(v >= 0, v.astype(np.uint64), np.uint64(P) - (-v).astype(np.uint64)).astype(np.uint64)


def fp_sub(a, b):
    """(a - b) mod p for canonical u64 arrays."""
    return np.where(a >= b, a - b, a + (np.uint64(P) - b)).astype(np.uint64)


def pack_pair(inp, out, k):
    """Canonical Fp of in + 2^k out for small signed integers (exact in int64)."""
    return emb(np.asarray(inp, np.int64) + (np.asarray(out, np.int64) << k))


def fp2_mul(a, b):
    a0, a1, b0, b1 = (int(x) for x in (a[0], a[1], b[0], b[1]))
    return ((a0 * b0 + 7 * a1 * b1) % P, (a0 * b1 + a1 * b0) % P)


def lift(col):
    x = np.zeros((col.size, 2), dtype=np.uint64)
    x[:, 0] = col
    return x


class Schedule:
    """The layer schedule over t proof rows at positions t0 .. t0 + t - 1
    attending over s = t0 + t keys (block_proof.rs BandShape: q = t; the
    prefill is the square band t0 = 0, a decode band has t0 > 0 and its own
    transcript and mask domains, chunk >= 1)."""

    def __init__(self, o, luts, t, t0=0, chunk=0):
        self.o, self.luts, self.t, self.t0, self.chunk = o, luts, t, t0, chunk
        self.s = t0 + t
        self.tp, self.sp = pow2(t), pow2(self.s)
        self.rect = HEAD_PAD * self.tp * self.sp
        exp = luts["exp"]
        assert exp[0x8000] == 0
        u = np.arange(1 << 16)
        self.gap_exp = np.where(u <= 0x8000, exp[((-u) & 0xFFFF)], 0).astype(np.int64)
        r = np.arange(1 << RECIP_BITS, dtype=np.int64)
        den = (r << 6) + 32
        hi = np.minimum(((1 << 26) + den // 2) // den, 32767)
        self.recip18 = np.where(r < (1 << 16), luts["softmax_recip"][np.minimum(r, 65535)], hi).astype(np.int64)

    # ---- lookup instances -------------------------------------------------
    def dom(self, layer, site):
        return site_domain(layer, site, self.chunk)

    def logup(self, f, table, mult, seed, layer, site):
        return self.o.logup_prove_fp(f, table, mult, seed, self.dom(layer, site))

    def range_site(self, acc, out, rows, cols, row_pad, col_pad, shift, seed, layer, site):
        half = 1 << (shift - 1)
        acc = np.asarray(acc, np.int64).reshape(rows, cols)
        out = np.asarray(out, np.int64).reshape(rows, cols)
        rem = np.full((row_pad, col_pad), half, dtype=np.int64)
        rem[:rows, :cols] = acc + half - (out << shift)
        assert rem.min() >= 0 and rem.max() < (1 << shift)
        rem = rem.reshape(-1)
        mult = np.bincount(rem, minlength=1 << shift).astype(np.uint32)
        return self.logup(rem.astype(np.uint64), np.arange(1 << shift, dtype=np.uint64), mult, seed, layer, site)

    def pair_site(self, inp, out, rows, cols, row_pad, col_pad, pad_in, pad_out, lut, signed, seed, layer, site):
        ic = np.full((row_pad, col_pad), pad_in, dtype=np.int64)
        oc = np.full((row_pad, col_pad), pad_out, dtype=np.int64)
        ic[:rows, :cols] = np.asarray(inp, np.int64).reshape(rows, cols)
        oc[:rows, :cols] = np.asarray(out, np.int64).reshape(rows, cols)
        ic, oc = ic.reshape(-1), oc.reshape(-1)
        f = pack_pair(ic, oc, 16)
        idx = (ic & 0xFFFF) if signed else ic
        mult = np.bincount(idx, minlength=1 << 16).astype(np.uint32)
        u = np.arange(1 << 16, dtype=np.int64)
        tin = u.astype(np.uint16).view(np.int16).astype(np.int64) if signed else u
        table = pack_pair(tin, lut, 16)
        return self.logup(f, table, mult, seed, layer, site)

    # ---- sumchecks ------------------------------------------------------------
    def product(self, a, b, tx):
        o = self.o
        n = a.shape[0]
        k = n.bit_length() - 1
        r = [tx.next_fp2() for _ in range(k)]
        words = []
        for j in range(k):
            words.append(o.product_round(a, b, a.shape[0] // 2))
            a = o.fold_rows(a, 1, a.shape[0], r[j])
            b = o.fold_rows(b, 1, b.shape[0], r[j])
        words.append(np.concatenate([a, b]))
        return np.concatenate(words)

    def triple(self, a, b, c, tx):
        o = self.o
        n = a.shape[0]
        k = n.bit_length() - 1
        r = [tx.next_fp2() for _ in range(k)]
        words = []
        for j in range(k):
            words.append(o.triple_product_round(a, b, c, a.shape[0] // 2))
            a, b, c = (o.fold_rows(x, 1, x.shape[0], r[j]) for x in (a, b, c))
        words.append(np.concatenate([a, b, c]))
        return np.concatenate(words)

    def eq(self, pt):
        pts = np.array(pt, dtype=np.uint64).reshape(-1, 2)
        return self.o.eq_rows(np.ascontiguousarray(pts), 1, len(pt)) if len(pt) else np.array([[1, 0]], np.uint64)

    def gemm(self, x, w, acc, m, k, n, seed, layer, site):
        o = self.o
        tx = o.FpStream(seed, self.dom(layer, site))
        m_pad, n_pad, k_pad = pow2(m), pow2(n), pow2(k)
        rj = [tx.next_fp2() for _ in range(n_pad.bit_length() - 1)]
        ri = [tx.next_fp2() for _ in range(m_pad.bit_length() - 1)]
        eq_j, eq_i = self.eq(rj), self.eq(ri)
        acc_r = o.matrix_fold(np.ascontiguousarray(acc, np.int64).reshape(-1), eq_i, m, n, 0, n, n_pad, 1, 0)
        claim = (0, 0)
        for j in range(n_pad):
            t = fp2_mul(acc_r[j], eq_j[j])
            claim = ((claim[0] + t[0]) % P, (claim[1] + t[1]) % P)
        a = o.matrix_fold(np.ascontiguousarray(x, np.int16).reshape(-1), eq_i, m, k, 0, k, k_pad, 0, 0)
        b = o.matrix_fold(np.ascontiguousarray(w, np.int16).reshape(-1), eq_j, k, n, 0, n, k_pad, 0, 1)
        return np.concatenate([np.array([claim], np.uint64), self.product(a, b, tx)])

    def ln_product(self, x, mean, rout, gain, seed, layer, site):
        t, tp, d = self.t, self.tp, np.asarray(gain).size
        tx = self.o.FpStream(seed, self.dom(layer, site))
        dp = pow2(d)
        xx = np.zeros((tp, dp), np.int64)
        xx[:t, :d] = np.asarray(x, np.int64).reshape(t, d)
        cen = np.zeros((tp, dp), np.int64)
        cen[:t] = xx[:t] - np.asarray(mean, np.int64)[:, None]
        rs = np.zeros(tp, np.int64)
        rs[:t] = np.asarray(rout, np.int64)
        g = np.zeros(dp, np.int64)
        g[:d] = np.asarray(gain, np.int64)
        return self.product(lift(emb(cen.reshape(-1))), lift(emb((rs[:, None] * g[None, :]).reshape(-1))), tx)

    # ---- one layer --------------------------------------------------------------
    def layer(self, r, lw, seed, layer, kv=None):
        """The words of one layer from the wires r (forward_layer names; a
        band_witness layer for a band) and, for a band, kv = (K, V) of all s
        cached rows (the prefill uses r's own K and V)."""
        t, tp, rect, t0, s, sp = self.t, self.tp, self.rect, self.t0, self.s, self.sp
        k_all, v_all = kv if kv is not None else (r["k"], r["v"])
        d = np.asarray(lw["ln1_gain"]).size
        dff, h = np.asarray(lw["ffn_up"]).size // d, d // DH
        assert h <= HEAD_PAD
        dp, fp, qp = pow2(d), pow2(dff), pow2(3 * d)
        lut = self.luts
        words = []
        words.append(self.range_site(r["ffn_down_acc"], r["ffn_down_q"], t, d, tp, dp, 10, seed, layer, "down_range"))
        words.append(self.pair_site(r["ffn_up_q"], r["gelu_out"], t, dff, tp, fp, 0, int(lut["gelu"][0]),
                                    lut["gelu"], True, seed, layer, "gelu"))
        words.append(self.range_site(r["ffn_up_acc"], r["ffn_up_q"], t, dff, tp, fp, 10, seed, layer, "up_range"))
        words.append(self.range_site(r["ln2_acc"], r["ln2_out"], t, d, tp, dp, 16, seed, layer, "ln2_norm"))
        words.append(self.pair_site(r["ln2_rsqrt_in"], r["ln2_rsqrt_out"], 1, t, 1, tp, 0, int(lut["ln_rsqrt"][0]),
                                    lut["ln_rsqrt"], False, seed, layer, "ln2_rsqrt"))
        words.append(self.range_site(r["proj_acc"], r["attn_proj_q"], t, d, tp, dp, 10, seed, layer, "proj_range"))
        words.append(self.range_site(r["av_acc"], r["av_q"], t, d, tp, dp, 12, seed, layer, "av_range"))
        # softmax columns over the padded packed rectangle (row i: window t0 + i + 1)
        caus = t * t0 + t * (t + 1) // 2
        packed = h * caus
        rs = np.asarray(r["row_shift"], np.int64).reshape(h, t)
        rc = np.asarray(r["recips"], np.int64).reshape(h, t)
        heads = np.repeat(np.arange(h), caus)
        rows = np.concatenate([np.repeat(np.arange(t), t0 + np.arange(1, t + 1))] * h)
        sq = np.asarray(r["scores_q"], np.int64)
        ex = np.asarray(r["exp_out"], np.int64)
        wt = np.asarray(r["weights"], np.int64)
        gap = np.zeros(rect, np.int64)
        gap[:packed] = rs[heads, rows] - sq
        exc = np.full(rect, self.gap_exp[0], np.int64)
        exc[:packed] = ex
        rem = np.full(rect, 1 << 13, np.int64)
        rem[:packed] = ex * rc[heads, rows] + (1 << 13) - (wt << 14)
        rcc = np.zeros(rect, np.int64)
        rcc[:packed] = rc[heads, rows]
        mask = np.zeros(rect, np.uint64)
        mask[:packed] = 1
        assert gap.min() >= 0 and gap.max() < 65536 and rem.min() >= 0 and rem.max() < (1 << 14)
        words.append(self.logup(rem.astype(np.uint64), np.arange(1 << 14, dtype=np.uint64),
                                np.bincount(rem, minlength=1 << 14).astype(np.uint32), seed, layer, "norm_range"))
        u = np.arange(1 << 16, dtype=np.int64)
        words.append(self.logup(pack_pair(gap, exc, 16), pack_pair(u, self.gap_exp, 16),
                                np.bincount(gap, minlength=1 << 16).astype(np.uint32), seed, layer, "exp"))
        rin = np.full((HEAD_PAD, tp), RECIP_PAD_INPUT, np.int64)
        rout = np.full((HEAD_PAD, tp), self.recip18[RECIP_PAD_INPUT], np.int64)
        rin[:h, :t] = np.asarray(r["denoms"], np.int64).reshape(h, t) >> 6
        rout[:h, :t] = rc
        rin, rout = rin.reshape(-1), rout.reshape(-1)
        v = np.arange(1 << RECIP_BITS, dtype=np.int64)
        words.append(self.logup(pack_pair(rin, rout, RECIP_BITS), pack_pair(v, self.recip18, RECIP_BITS),
                                np.bincount(rin, minlength=1 << RECIP_BITS).astype(np.uint32), seed, layer, "recip"))
        words.append(self.range_site(r["scores_acc"], r["scores_q"], 1, packed, 1, rect, 10, seed, layer,
                                     "scores_range"))
        words.append(self.range_site(r["qkv_acc"], np.asarray(r["qkv_q"]), t, 3 * d, tp, qp, 10, seed, layer,
                                     "qkv_range"))
        words.append(self.range_site(r["ln1_acc"], r["ln1_out"], t, d, tp, dp, 16, seed, layer, "ln1_norm"))
        words.append(self.pair_site(r["ln1_rsqrt_in"], r["ln1_rsqrt_out"], 1, t, 1, tp, 0, int(lut["ln_rsqrt"][0]),
                                    lut["ln_rsqrt"], False, seed, layer, "ln1_rsqrt"))
        # sumchecks
        o = self.o
        words.append(self.gemm(r["gelu_out"], lw["ffn_down"], r["ffn_down_acc"], t, dff, d, seed, layer, "gemm_down"))
        words.append(self.gemm(r["ln2_out"], lw["ffn_up"], r["ffn_up_acc"], t, d, dff, seed, layer, "gemm_up"))
        words.append(self.ln_product(r["attn_block_out"], r["ln2_mean"], r["ln2_rsqrt_out"], lw["ln2_gain"], seed, layer,
                                     "ln2_had"))
        words.append(self.gemm(r["av_q"], lw["attn_proj"], r["proj_acc"], t, d, d, seed, layer, "gemm_proj"))
        # A.V over (head, key position j < s): rows i with t0 + i >= j
        tx = o.FpStream(seed, self.dom(layer, "av"))
        rcp = [tx.next_fp2() for _ in range(6)]
        rh = [tx.next_fp2() for _ in range(4)]
        ri = [tx.next_fp2() for _ in range(tp.bit_length() - 1)]
        eq_c, eq_h, eq_i = self.eq(rcp), self.eq(rh), self.eq(ri)
        words.append(self.triple(*self.av_factors(wt, v_all, eq_i, eq_c, eq_h, h, d), tx))
        tx = o.FpStream(seed, self.dom(layer, "norm_had"))
        words.append(self.triple(lift(emb(exc)), lift(emb(rcc)), lift(mask), tx))
        # Q.K^T: the band's Q rows against all s cached K rows
        tx = o.FpStream(seed, self.dom(layer, "qk"))
        rj = [tx.next_fp2() for _ in range(sp.bit_length() - 1)]
        ri = [tx.next_fp2() for _ in range(tp.bit_length() - 1)]
        rh = [tx.next_fp2() for _ in range(4)]
        eq_i, eq_j, eq_h = self.eq(ri), self.eq(rj), self.eq(rh)
        qr = o.matrix_fold(np.ascontiguousarray(r["q"], np.int16).reshape(-1), eq_i, t, d, 0, d, dp, 0, 0)
        kr = o.matrix_fold(np.ascontiguousarray(k_all, np.int16).reshape(-1), eq_j, s, d, 0, d, dp, 0, 0)
        cc = np.ascontiguousarray(eq_h[np.arange(dp) // DH])
        words.append(self.triple(qr, kr, cc, tx))
        words.append(self.gemm(r["ln1_out"], lw["c_attn"], r["qkv_acc"], t, d, 3 * d, seed, layer, "gemm_qkv"))
        words.append(self.ln_product(r["x_in"], r["ln1_mean"], r["ln1_rsqrt_out"], lw["ln1_gain"], seed, layer,
                                     "ln1_had"))
        return np.concatenate([np.asarray(w, np.uint64).reshape(-1, 2) for w in words])

    def av_factors(self, wt, v_all, eq_i, eq_c, eq_h, h=H, d=D):
        """The A.V contraction's factors over (head, key position j < s):
        A = sum over the rows i with t0 + i >= j of eq_i[i] w[h,i,j] (band
        packing), B = sum_c eq_c[c] v[j, h*64 + c], C = eq_h[h]."""
        t, t0, s, sp = self.t, self.t0, self.s, self.sp
        caus = t * t0 + t * (t + 1) // 2
        wt = np.asarray(wt, np.int64)
        A = np.zeros((HEAD_PAD * sp, 2), np.uint64)
        B = np.zeros((HEAD_PAD * sp, 2), np.uint64)
        C = np.zeros((HEAD_PAD * sp, 2), np.uint64)
        vv = np.asarray(v_all, np.int64).reshape(s, d)
        for hh in range(HEAD_PAD):
            C[hh * sp:(hh + 1) * sp] = eq_h[hh]
            if hh >= h:
                continue
            wh = wt[hh * caus:(hh + 1) * caus]
            for j in range(s):
                ia = np.arange(max(0, j - t0), t)
                A[hh * sp + j] = _dot_base(eq_i[ia], wh[ia * t0 + ia * (ia + 1) // 2 + j])
                B[hh * sp + j] = _dot_base(eq_c[:64], vv[j, hh * 64:(hh + 1) * 64])
        return A, B, C

    def corrections(self, r, mac_seed, layer):
        """x - mask of the boundary wires (the proof's t rows); one mask domain
        per (chunk, layer, wire), row i at (tag << 32) | i."""
        out = []
        d = np.asarray(r["x_in"]).size // self.t
        for w, name in enumerate(("x_in", "k", "v", "attn_block_out", "ffn_block_out")):
            tag = (self.chunk << 16) | (layer * 8 + w)
            masks = self.o.chacha_fp_rows(mac_seed, tag << 32, self.t, d).reshape(-1)
            out.append(fp_sub(emb(np.asarray(r[name]).reshape(-1)), masks))
        return out


def _dot_base(eqs, vals):
    s0 = s1 = 0
    for e, v in zip(eqs, vals):
        v = int(v) % P
        if v:
            s0 += int(e[0]) * v
            s1 += int(e[1]) * v
    return (s0 % P, s1 % P)


def pcs_rows(total):
    """Rows of the weight matrix: 8192 (GPT2_FULL, ligero.rs:59-60) while the
    weights fit, else the power of two the weights fill (the MLE row
    variables are ceil(log2 rows) either way, ligero.rs:47-50, 66-68)."""
    cols = 1 << PCS_COL_BITS
    need = -(-total // cols)
    return max(PCS_ROWS, pow2(need))


def pcs_root(o, model, pad_seed):
    """The weight commitment: every layer's weights, then wte, wpe, final LN,
    row-major into pcs_rows rows of 2^14 int16 (8192 for GPT-2 small), 512
    ChaCha8 pads per row, RS code 2^15, BLAKE3 column tree."""
    cols, code_len = 1 << PCS_COL_BITS, 1 << PCS_CODE_BITS
    parts = []
    for lw in model.layers:
        parts += [lw[k].reshape(-1) for k in ("c_attn", "attn_proj", "ffn_up", "ffn_down", "ln1_gain", "ln1_bias",
                                              "ln2_gain", "ln2_bias")]
    parts += [model.wte.reshape(-1), model.wpe.reshape(-1), model.lnf_gain, model.lnf_bias]
    flat = np.concatenate(parts).astype(np.int16)
    rows = pcs_rows(flat.size)
    w = np.zeros(rows * cols, np.int16)
    w[:flat.size] = flat
    pads = o.chacha_fp_rows(pad_seed, 0, rows, PCS_PAD)
    msgs = o.pcs_messages(w, np.ascontiguousarray(pads), rows, cols, PCS_PAD, code_len)
    code = o.ntt_batch(msgs.reshape(rows, code_len)[:, :cols + PCS_PAD].copy(), rows, cols + PCS_PAD, code_len)
    tree = o.merkle_tree(o.hash_fp_columns(code, rows, code_len))
    return bytes(tree[-1])
