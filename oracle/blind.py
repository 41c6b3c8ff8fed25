"""Oracle (test infrastructure only): blind LogUp corrections and the
VOLE-MAC correlation keys of the reference's mock correlation backend.

Blind LogUp sink (rust/volta-proto/src/logup.rs:1903-2000 BlindSink, and
the reference's own blind-rounds benchmark cuda/p7_logup_blind_rounds.cu:
185-215 blind_begin / blind_round / blind_finish, whose FNV checksum over
every round message, fold and correction is the golden
p7-gpu-logup-blind-rounds-*.json "all_rounds_checksum"):
  * root corrections  root_k - mask_k                     (k = p, q)
  * per round j       h0 = cpref (lambda pq0 + qq0), h2 = cpref (lambda pq2 + qq2)
                      corrections (h0 - mask_j0, h2 - mask_j1);
                      cpref <- cpref * eq(point_j, r_j)   (2 p r + 1 - p - r)
  * split corrections split_k - mask_k                    (p0, p1, q0, q1)
  * product corrections (p0 q1, p1 q0, q0 q1) - masks.

Mock correlations (rust/volta-mac/src/corr.rs, ProverBackend::Mock):
  * full-field draw at dom: x_k = FpStream(seed, dom | FULL_BIT).next_fp2(),
    tag m_k = FpStream(seed, dom | FULL_BIT | TAG_BIT).next_fp2()
    (draw_fulls, 1930-1978), verifier key m_k + delta x_k (2480-2486);
  * subfield draw at dom: masks r_k = FpStream(seed, dom).next_fp(), prover
    tags FpStream(seed, dom | TAG_BIT).next_fp2() (draw_sub_tags,
    1896-1915), verifier keys k_r = m_k + delta r_k (2354-2357) and, for a
    correction c, k = k_r + delta c (auth_verifier, auth.rs:35-53): the
    MAC relation k = m + delta x of the authenticated value x = r + c.

Imported by tests/ only.
"""

from __future__ import annotations

import numpy as np

P = 0xFFFFFFFF00000001
TAG_BIT = 1 << 63
FULL_BIT = 1 << 62
FNV_PRIME = 0x00000100000001B3
M64 = (1 << 64) - 1


def f2(x):
    return (int(x[0]) % P, int(x[1]) % P)


def add(a, b):
    return ((a[0] + b[0]) % P, (a[1] + b[1]) % P)


def sub(a, b):
    return ((a[0] - b[0]) % P, (a[1] - b[1]) % P)


def mul(a, b):
    return ((a[0] * b[0] + 7 * a[1] * b[1]) % P, (a[0] * b[1] + a[1] * b[0]) % P)


def eq_step(p, r):
    pr = mul(p, r)
    return sub(add(add(pr, pr), (1, 0)), add(p, r))


# ---- the blind sink's corrections --------------------------------------------

def blind_artifacts(accs, splits, inp):
    """accs: per round the 4 raw accumulators (pq0, pq2, qq0, qq2) of the
    general LogUp round; splits: the 4 final values (p0, p1, q0, q1);
    inp: roots, root_masks, lambda, points, round_masks, split_masks,
    prod_masks, challenges.  Returns the correction artifacts."""
    art = {"root": [sub(f2(inp["roots"][k]), f2(inp["root_masks"][k])) for k in range(2)], "rounds": []}
    lam, cpref = f2(inp["lambda"]), (1, 0)
    for j, acc in enumerate(accs):
        pq0, pq2, qq0, qq2 = (f2(a) for a in acc)
        h0 = mul(cpref, add(mul(lam, pq0), qq0))
        h2 = mul(cpref, add(mul(lam, pq2), qq2))
        m = inp["round_masks"][j]
        art["rounds"].append([sub(h0, f2(m[0])), sub(h2, f2(m[1]))])
        cpref = mul(cpref, eq_step(f2(inp["points"][j]), f2(inp["challenges"][j])))
    s = [f2(x) for x in splits]
    art["split"] = [sub(s[k], f2(inp["split_masks"][k])) for k in range(4)]
    prods = [mul(s[0], s[3]), mul(s[1], s[2]), mul(s[2], s[3])]
    art["prod"] = [sub(prods[k], f2(inp["prod_masks"][k])) for k in range(3)]
    return art


def golden_inputs(log2n: int) -> dict:
    """The closed-form blind inputs of the reference's benchmark
    (cuda/p7_logup_blind_rounds.cu:335-365)."""
    return {
        "roots": [(701, 907), (1103, 1301)],
        "root_masks": [(1709, 1901), (2203, 2503)],
        "lambda": (2707, 2903),
        "points": [(3109 + 12 * j, 3301 + 14 * j) for j in range(log2n)],
        "round_masks": [[(3701 + 20 * j, 3907 + 22 * j), (4201 + 24 * j, 4409 + 26 * j)] for j in range(log2n)],
        "split_masks": [(4703 + 30 * i, 5003 + 32 * i) for i in range(4)],
        "prod_masks": [(5303 + 34 * i, 5501 + 36 * i) for i in range(3)],
        "challenges": [(101 + 2 * j, 211 + 3 * j) for j in range(log2n)],
    }


def fnv_fp2(h: int, x) -> int:
    h = ((h ^ (int(x[0]) & M64)) * FNV_PRIME) & M64
    return ((h ^ (int(x[1]) & M64)) * FNV_PRIME) & M64


def hash_artifacts(h: int, art) -> int:
    for x in art["root"]:
        h = fnv_fp2(h, x)
    for row in art["rounds"]:
        for x in row:
            h = fnv_fp2(h, x)
    for x in art["split"] + art["prod"]:
        h = fnv_fp2(h, x)
    return h


# ---- mock correlations: masks, tags, verifier keys -----------------------------

def full_corrs(o, seed: bytes, dom: int, n: int):
    """(x_k, m_k) of a full-field draw at dom."""
    xs, ms = o.FpStream(seed, dom | FULL_BIT), o.FpStream(seed, dom | FULL_BIT | TAG_BIT)
    return [(xs.next_fp2(), ms.next_fp2()) for _ in range(n)]


def full_keys(o, seed: bytes, dom: int, n: int, delta):
    return [add(m, mul(f2(delta), x)) for x, m in full_corrs(o, seed, dom, n)]


def sub_masks(o, seed: bytes, dom: int, n: int):
    s = o.FpStream(seed, dom)
    return [s.next_fp() for _ in range(n)]


def sub_tags(o, seed: bytes, dom: int, n: int):
    """draw_sub_tags: the prover's MAC tags of a subfield draw at dom."""
    s = o.FpStream(seed, dom | TAG_BIT)
    return [s.next_fp2() for _ in range(n)]


def auth_verifier(o, seed: bytes, dom: int, corr, delta):
    """Verifier keys of a correction batch at dom: m + delta (r + c)."""
    tags = sub_tags(o, seed, dom, len(corr))
    masks = sub_masks(o, seed, dom, len(corr))
    d = f2(delta)
    return [add(add(m, (d[0] * r % P, d[1] * r % P)), (d[0] * int(c) % P, d[1] * int(c) % P))
            for m, r, c in zip(tags, masks, corr)]


def mac_holds(tags, keys, values, delta) -> bool:
    """k = m + delta x for every authenticated value x (canonical Fp)."""
    d = f2(delta)
    return all(k == add(f2(m), (d[0] * int(x) % P, d[1] * int(x) % P)) for m, k, x in zip(tags, keys, values))


# ---- the blind LogUp prover, its transcript and its wire format ---------------

TX_CONTEXT = "volta-zk/transcript/canonical-moves/v1"
U64_MAX = (1 << 64) - 1


class Transcript:
    """Private seeded transcript (rust/volta-mac/src/transcript.rs): challenges
    from FpStream(seed, u64::MAX) (84-110); every message charged to a label
    (account, 358-361) and bound as kind || u16 label length || label || u64
    length || message into the canonical move stream (append_message
    215-233; challenge requests 3 || 2 for Fp2, 3 || 1 for Fp, 3 || 3 || width
    for bits, 362-380), whose BLAKE3 derive-key hash with the context
    "volta-zk/transcript/canonical-moves/v1" is the binding digest (654-667)."""

    def __init__(self, o, seed: bytes):
        self.o, self.chal, self.moves, self.ledger = o, o.FpStream(seed, U64_MAX), bytearray(), {}

    def append_message(self, label: str, msg: bytes):
        self.ledger[label] = self.ledger.get(label, 0) + len(msg)
        lb = label.encode()
        self.moves += bytes([1]) + len(lb).to_bytes(2, "little") + lb + len(msg).to_bytes(8, "little") + msg

    def append_fp2s(self, label: str, values):
        self.append_message(label, b"".join(wire_fp2(v) for v in values))

    def challenge_fp2(self):
        self.moves += bytes([3, 2])
        return self.chal.next_fp2()

    def digest(self) -> bytes:
        return self.o.blake3_derive_key(TX_CONTEXT, bytes(self.moves))

    def total_bytes(self) -> int:
        return sum(self.ledger.values())


def wire_fp2(v) -> bytes:
    return int(v[0]).to_bytes(8, "little") + int(v[1]).to_bytes(8, "little")


def encode_blind_frac(root_corrs, layers) -> bytes:
    """BlindFracProof { root_corrs: [Fp2; 2], layers: Vec<BlindLayerProof>,
    aux: Option<BlindAuxPart> } under model_proof_codec.rs's Wire rules
    (rust/volta-proto/src/model_proof_codec.rs:202-320, 362-364): fixed arrays
    without a length, Vec as u32 LE length + items, Option None as byte 0."""
    out = b"".join(wire_fp2(x) for x in root_corrs) + len(layers).to_bytes(4, "little")
    for rounds, split, z in layers:
        out += len(rounds).to_bytes(4, "little") + b"".join(wire_fp2(a) + wire_fp2(b) for a, b in rounds)
        out += b"".join(wire_fp2(x) for x in split) + b"".join(wire_fp2(x) for x in z)
    return out + b"\x00"


def blind_logup_prove(o, f, table, mult, tx_seed: bytes, corr_seed: bytes, dom_base: int):
    """blind_logup_prove (rust/volta-proto/src/logup.rs:3184-3225) with a fresh
    Transcript::new(tx_seed) and the mock CorrelationStream::new(corr_seed):
    the clear messages are the oracle's clear LogUp proof under the same
    private challenge stream (the sinks draw alpha, then per layer lambda, the
    round challenges and the split challenge in the same order); BlindSink
    (1927-2004) publishes each as its correction against the full-field masks
    of one fresh domain per root / round / split / product group, and
    cross_prover (2526-2556) the corrections of p_f q_t, p_t q_f, 1/q_f, 1/q_t.
    Returns (BlindLogupProof wire bytes, transcript digest, transcript bytes,
    the domain cursor after the proof)."""
    words = o.logup_prove(f, table, mult, tx_seed, U64_MAX)
    w = [tuple(int(x) for x in row) for row in words]
    tx = Transcript(o, tx_seed)
    assert tx.challenge_fp2() == w[0]
    dom = dom_base
    pos = 1
    out, roots = b"", []
    for n in (len(f), len(table)):
        depth = n.bit_length() - 1
        root = (w[pos], w[pos + 1])
        pos += 2
        roots.append(root)
        m = [x for x, _ in full_corrs(o, corr_seed, dom, 2)]
        dom += 1
        root_corrs = [sub(root[0], m[0]), sub(root[1], m[1])]
        tx.append_fp2s("logup_root_corrections", root_corrs)
        layers = []
        for layer in range(depth):
            tx.challenge_fp2()  # lambda
            rounds = []
            for _ in range(layer):
                m = [x for x, _ in full_corrs(o, corr_seed, dom, 2)]
                dom += 1
                c = (sub(w[pos], m[0]), sub(w[pos + 1], m[1]))
                pos += 2
                tx.append_fp2s("logup_round_corrections", c)
                rounds.append(c)
                tx.challenge_fp2()  # round challenge
            s = w[pos:pos + 4]
            pos += 4
            m = [x for x, _ in full_corrs(o, corr_seed, dom, 4)]
            dom += 1
            split = [sub(s[k], m[k]) for k in range(4)]
            tx.append_fp2s("logup_split_corrections", split)
            zx = [mul(s[0], s[3]), mul(s[1], s[2]), mul(s[2], s[3])]
            m = [x for x, _ in full_corrs(o, corr_seed, dom, 3)]
            dom += 1
            z = [sub(zx[k], m[k]) for k in range(3)]
            tx.append_fp2s("logup_prod_corrections", z)
            tx.challenge_fp2()  # split challenge
            layers.append((rounds, split, z))
        out += encode_blind_frac(root_corrs, layers)
    assert pos == len(w)
    (pf, qf), (pt, qt) = roots
    zx = [mul(pf, qt), mul(pt, qf), f2(o.fp2_inv(qf)), f2(o.fp2_inv(qt))]
    m = [x for x, _ in full_corrs(o, corr_seed, dom, 4)]
    dom += 1
    cross = [sub(zx[k], m[k]) for k in range(4)]
    tx.append_fp2s("logup_cross_corrections", cross)
    out += b"".join(wire_fp2(x) for x in cross)
    return out, tx.digest(), tx.total_bytes(), dom
