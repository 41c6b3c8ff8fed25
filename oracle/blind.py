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
