"""CPU stand-in for one shard's device work (test infrastructure): the same
outputs as vzh_triple_sumcheck on a slice and vzh_logup_local, computed with
the oracle, so the host-side combination (volta_zk_b200/sharded.py) and the
gloo all-gather path can be checked without a GPU."""

import numpy as np

P = 0xFFFFFFFF00000001


def side_draws(depth: int) -> int:
    return sum(l + 2 for l in range(depth))


def side_schedule(ch, depth: int):
    """Per layer: lambda, l round challenges, split challenge; claim points."""
    lam, r, t, point = [], [], [], [[] for _ in range(depth)]
    pos = 0
    for l in range(depth):
        lam.append(ch[pos])
        r.append(list(ch[pos + 1:pos + 1 + l]))
        t.append(ch[pos + 1 + l])
        pos += l + 2
        if l + 1 < depth:
            point[l + 1] = [t[l]] + r[l]
    return lam, r, t, point


def triple_local(oracle, a, b, c, seed):
    """Messages of the slice's own rounds and its three final values."""
    n = a.shape[0]
    k = n.bit_length() - 1
    s = oracle.FpStream(seed, 2**64 - 1)
    msgs = []
    cur = [a.copy(), b.copy(), c.copy()]
    for _ in range(k):
        msgs.append(oracle.triple_product_round(*cur, cur[0].shape[0] // 2))
        r = s.next_fp2()
        cur = [oracle.fold_rows(x, 1, x.shape[0], r) for x in cur]
    m = np.concatenate(msgs) if msgs else np.zeros((0, 2), np.uint64)
    return m, np.concatenate([x[:1] for x in cur])


def _side(oracle, col, mult, s_bits, alpha, sched, neg):
    lam, r, _, point = sched
    n = col.shape[0]
    depth = (n.bit_length() - 1) + s_bits
    leaf = np.array([(alpha[0] - int(v)) % P for v in col], dtype=np.uint64)
    tp, tq = oracle.logup_tree(leaf, mult, n, alpha[1], neg)
    words = [tp[0], tq[0]]
    for l in range(s_bits, depth):
        L = l - s_bits
        if l + 1 == depth:
            cp, cq = oracle.materialize_leaves(leaf, mult, n, alpha[1], neg)
        else:
            off = (2 << L) - 1
            cp, cq = tp[off:off + (2 << L)], tq[off:off + (2 << L)]
        vec = [np.ascontiguousarray(x) for x in (cp[0::2], cp[1::2], cq[0::2], cq[1::2])]
        pt = np.array(point[l][:L], dtype=np.uint64).reshape(-1, 2)
        suffix = oracle.suffix_eq(pt) if L else None
        for j in range(L):
            soff = (1 << (L - 1 - j)) - 1
            acc = oracle.logup_general_round(*vec, np.ascontiguousarray(suffix[soff:]), vec[0].shape[0] // 2)
            words.extend(acc)
            vec = [oracle.fold_rows(v, 1, v.shape[0], r[l][j]) for v in vec]
        words.extend(v[0] for v in vec)
    return words


def logup_local(oracle, f_slice, t_slice, mult_slice, s_bits, seed, domain):
    """f_slice / t_slice: canonical Fp columns of this shard."""
    df = (f_slice.shape[0].bit_length() - 1) + s_bits
    dt = (t_slice.shape[0].bit_length() - 1) + s_bits
    st = oracle.FpStream(seed, domain)
    total = 1 + side_draws(df) + side_draws(dt)
    ch = [st.next_fp2() for _ in range(total)]
    alpha = ch[0]
    words = [np.array(alpha, dtype=np.uint64)]
    sf = side_schedule(ch[1:1 + side_draws(df)], df)
    stt = side_schedule(ch[1 + side_draws(df):], dt)
    words += _side(oracle, f_slice, None, s_bits, alpha, sf, False)
    words += _side(oracle, t_slice, mult_slice, s_bits, alpha, stt, True)
    return np.array([np.asarray(w, dtype=np.uint64).reshape(2) for w in words], dtype=np.uint64), ch


def embed_i16(v):
    v64 = v.astype(np.int64)
    return np.where(v64 >= 0, v64.astype(np.uint64), np.uint64(P) - (-v64).astype(np.uint64)).astype(np.uint64)
