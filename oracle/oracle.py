"""NumPy glue over the C oracle (``oracle/_build/liboracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` leg of ``bench.py`` as the checker.  The shipped
library never imports it.

Fp2 vectors are ``numpy.uint64`` arrays of shape ``(n, 2)`` (c0, c1), the
same 16-byte ``Fp2Repr`` layout the reference seam uses
(rust/volta-accel/src/lib.rs:394-399).
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
P = 0xFFFFFFFF00000001

_lib = None


def reference_cuda_dir() -> str:
    """The reference's ``cuda/`` directory, when its source tree is present:
    ``$VOLTA_REFERENCE_DIR/cuda``, else a ``reference`` checkout beside this
    repository.  Empty when neither exists (the GPU box has no reference)."""
    root = os.environ.get("VOLTA_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                                 "reference")
    d = os.path.join(root, "cuda")
    return d if os.path.isdir(d) else ""


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE, f"REF_DIR={reference_cuda_dir()}"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


class Fp2C(C.Structure):
    _fields_ = [("c0", C.c_uint64), ("c1", C.c_uint64)]


class Stream(C.Structure):
    _fields_ = [
        ("key", C.c_uint32 * 8),
        ("stream", C.c_uint64),
        ("block", C.c_uint64),
        ("words", C.c_uint32 * 16),
        ("idx", C.c_uint32),
    ]


_vp = C.c_void_p
_sz = C.c_size_t
_u64 = C.c_uint64


def _declare(L):
    L.or_fp_mul.restype = _u64
    L.or_fp_mul.argtypes = [_u64, _u64]
    L.or_fp_add.restype = _u64
    L.or_fp_add.argtypes = [_u64, _u64]
    L.or_fp_sub.restype = _u64
    L.or_fp_sub.argtypes = [_u64, _u64]
    L.or_fp_pow.restype = _u64
    L.or_fp_pow.argtypes = [_u64, _u64]
    L.or_fp_inv.restype = _u64
    L.or_fp_inv.argtypes = [_u64]
    L.or_fp2_mul.restype = Fp2C
    L.or_fp2_mul.argtypes = [Fp2C, Fp2C]
    L.or_fp2_inv.restype = Fp2C
    L.or_fp2_inv.argtypes = [Fp2C]
    L.or_fp_mul_batch.argtypes = [_vp, _vp, _vp, _sz]
    L.or_stream_init.argtypes = [C.POINTER(Stream), C.c_char_p, _u64]
    L.or_stream_next_u64.restype = _u64
    L.or_stream_next_u64.argtypes = [C.POINTER(Stream)]
    L.or_stream_next_fp.restype = _u64
    L.or_stream_next_fp.argtypes = [C.POINTER(Stream)]
    L.or_stream_next_fp2.restype = Fp2C
    L.or_stream_next_fp2.argtypes = [C.POINTER(Stream)]
    L.or_stream_next_bits.restype = _u64
    L.or_stream_next_bits.argtypes = [C.POINTER(Stream), C.c_uint]
    L.or_stream_fill_u64.argtypes = [C.c_char_p, _u64, _sz, _vp]
    L.or_chacha_fp_rows.argtypes = [C.c_char_p, _u64, _sz, _sz, _vp]
    L.or_chacha_fp2_rows_padded.argtypes = [C.c_char_p, _u64, _sz, _sz, _sz, _vp]
    L.or_product_round.argtypes = [_vp, _vp, _sz, _vp]
    L.or_triple_product_round.argtypes = [_vp, _vp, _vp, _sz, _vp]
    L.or_logup_general_round.argtypes = [_vp, _vp, _vp, _vp, _vp, _sz, _vp]
    L.or_fold_rows.argtypes = [_vp, _sz, _sz, Fp2C, _vp]
    L.or_logup_tree.argtypes = [_vp, _vp, _sz, _u64, C.c_int, _vp, _vp]
    L.or_materialize_leaves.argtypes = [_vp, _vp, _sz, _u64, C.c_int, _vp, _vp]
    L.or_suffix_eq.argtypes = [_vp, _sz, _vp]
    L.or_eq_rows.argtypes = [_vp, _sz, _sz, _vp]
    L.or_eq_vec.argtypes = [_vp, _sz, _vp]
    L.or_aux_round.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz,
                               Fp2C, Fp2C, Fp2C, _vp]
    L.or_matrix_fold.argtypes = [_vp, _vp, _sz, _sz, _sz, _sz, _sz, C.c_int, C.c_int, _vp]
    L.or_triple_sumcheck.argtypes = [_vp, _vp, _vp, _sz, C.c_char_p, _vp, _vp]
    L.or_logup_prove.restype = _sz
    L.or_logup_prove.argtypes = [_vp, _sz, _vp, _sz, _vp, C.c_char_p, _u64, _vp, _sz]
    L.or_logup_prove_fp.restype = _sz
    L.or_logup_prove_fp.argtypes = [_vp, _sz, _vp, _sz, _vp, C.c_char_p, _u64, _vp, _sz]
    L.or_ntt_batch.argtypes = [_vp, _sz, _sz, _sz, _vp]
    L.or_ntt_fp2_batch.argtypes = [_vp, _sz, _sz, _sz, _vp]
    L.or_blake3.argtypes = [_vp, _sz, _vp]
    L.or_blake3_derive_key.argtypes = [_vp, _sz, _vp, _sz, _vp]
    L.or_hash_fp_columns.argtypes = [_vp, _sz, _sz, _vp]
    L.or_hash_fp2_columns.argtypes = [_vp, _sz, _sz, _vp]
    L.or_merkle_tree.argtypes = [_vp, _sz, _vp]
    L.or_merkle_paths.argtypes = [_vp, _sz, _vp, _sz, _vp]
    L.or_pcs_messages.argtypes = [_vp, _vp, _sz, _sz, _sz, _sz, _vp]
    L.or_pcs_combine_rows.argtypes = [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _vp]
    L.or_gemm_i64.argtypes = [_vp, _vp, _vp, _sz, _sz, _sz]
    L.or_gemm_requant_auth.argtypes = [_vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, C.c_uint32]
    L.or_set_threads.argtypes = [C.c_int]
    L.or_max_threads.restype = C.c_int
    L.or_fnv_u64.restype = _u64
    L.or_fnv_u64.argtypes = [_u64, _vp, _sz]


def host_threads() -> int:
    """Host cores this process may run on (affinity mask / cgroup cpuset)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def set_threads(n: int) -> int:
    """Pin the oracle's OpenMP thread count; returns the count now in force."""
    lib().or_set_threads(int(n))
    return int(lib().or_max_threads())


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(_vp)


def fp2(x) -> Fp2C:
    return Fp2C(int(x[0]) % P, int(x[1]) % P)


def fp2_tuple(v: Fp2C):
    return (v.c0, v.c1)


def fp2_array(n: int) -> np.ndarray:
    return np.zeros((n, 2), dtype=np.uint64)


# ---- field ----------------------------------------------------------------

def fp_mul(a: int, b: int) -> int:
    return lib().or_fp_mul(a, b)


def fp2_mul(a, b):
    return fp2_tuple(lib().or_fp2_mul(fp2(a), fp2(b)))


def fp2_inv(a):
    return fp2_tuple(lib().or_fp2_inv(fp2(a)))


def fp_mul_batch(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint64)
    b = np.ascontiguousarray(b, dtype=np.uint64)
    out = np.empty_like(a)
    lib().or_fp_mul_batch(_p(a), _p(b), _p(out), a.size)
    return out


# ---- FpStream ---------------------------------------------------------------

class FpStream:
    """rust/volta-field/src/lib.rs:222-268 (FpStream::domain_separated)."""

    def __init__(self, seed: bytes, domain: int):
        assert len(seed) == 32
        self._s = Stream()
        lib().or_stream_init(C.byref(self._s), seed, domain & 0xFFFFFFFFFFFFFFFF)

    def next_u64(self) -> int:
        return lib().or_stream_next_u64(C.byref(self._s))

    def next_fp(self) -> int:
        return lib().or_stream_next_fp(C.byref(self._s))

    def next_fp2(self):
        return fp2_tuple(lib().or_stream_next_fp2(C.byref(self._s)))

    def next_bits(self, width: int) -> int:
        return lib().or_stream_next_bits(C.byref(self._s), width)


def stream_u64(seed: bytes, domain: int, n: int) -> np.ndarray:
    out = np.zeros(n, dtype=np.uint64)
    lib().or_stream_fill_u64(seed, domain & 0xFFFFFFFFFFFFFFFF, n, _p(out))
    return out


def chacha_fp_rows(seed: bytes, base: int, rows: int, count: int) -> np.ndarray:
    out = np.zeros((rows, count), dtype=np.uint64)
    lib().or_chacha_fp_rows(seed, base, rows, count, _p(out))
    return out


def chacha_fp2_rows_padded(seed: bytes, base: int, rows: int, count: int, padded: int):
    out = np.zeros((rows * padded, 2), dtype=np.uint64)
    lib().or_chacha_fp2_rows_padded(seed, base, rows, count, padded, _p(out))
    return out


# ---- sumcheck -----------------------------------------------------------------

def product_round(a, b, pairs):
    out = fp2_array(2)
    lib().or_product_round(_p(a), _p(b), pairs, _p(out))
    return out


def triple_product_round(a, b, c, pairs):
    out = fp2_array(3)
    lib().or_triple_product_round(_p(a), _p(b), _p(c), pairs, _p(out))
    return out


def logup_general_round(p0, p1, q0, q1, suffix, pairs):
    out = fp2_array(4)
    lib().or_logup_general_round(_p(p0), _p(p1), _p(q0), _p(q1), _p(suffix), pairs, _p(out))
    return out


def fold_rows(x, rows, length, r):
    out = fp2_array(rows * (length // 2))
    lib().or_fold_rows(_p(x), rows, length, fp2(r), _p(out))
    return out


def logup_tree(leaf: np.ndarray, mult, n: int, alpha1: int, neg_mult: bool):
    p = fp2_array(n - 1)
    q = fp2_array(n - 1)
    mp = _p(mult) if mult is not None else None
    lib().or_logup_tree(_p(leaf), mp, n, alpha1, int(neg_mult), _p(p), _p(q))
    return p, q


def materialize_leaves(leaf, mult, n, alpha1, neg_mult):
    p = fp2_array(n)
    q = fp2_array(n)
    mp = _p(mult) if mult is not None else None
    lib().or_materialize_leaves(_p(leaf), mp, n, alpha1, int(neg_mult), _p(p), _p(q))
    return p, q


def suffix_eq(point: np.ndarray):
    L = point.shape[0]
    out = fp2_array((1 << L) - 1)
    lib().or_suffix_eq(_p(point), L, _p(out))
    return out


def eq_rows(points: np.ndarray, rows: int, dims: int):
    out = fp2_array(rows << dims)
    lib().or_eq_rows(_p(points), rows, dims, _p(out))
    return out


def aux_round(q0, q1, suffix, columns, eq, claim_cols, weights, column_count, claim_count,
              vector_len, lam, cpref, point):
    out = fp2_array(3)
    lib().or_aux_round(_p(q0), _p(q1), _p(suffix), _p(columns),
                       _p(eq) if eq is not None else None,
                       _p(claim_cols) if claim_cols is not None else None,
                       _p(weights) if weights is not None else None,
                       column_count, claim_count, vector_len,
                       fp2(lam), fp2(cpref), fp2(point), _p(out))
    return out


def matrix_fold(inp, weights, rows, stride, column_offset, cols, out_pad, kind, axis):
    out = fp2_array(out_pad)
    lib().or_matrix_fold(_p(inp), _p(weights), rows, stride, column_offset, cols, out_pad,
                         kind, axis, _p(out))
    return out


def triple_sumcheck(a, b, c, chal_seed: bytes):
    a = a.copy(); b = b.copy(); c = c.copy()
    n = a.shape[0]
    rounds = n.bit_length() - 1
    msgs = fp2_array(3 * rounds)
    finals = fp2_array(3)
    lib().or_triple_sumcheck(_p(a), _p(b), _p(c), n, chal_seed, _p(msgs), _p(finals))
    return msgs, finals


def logup_prove_words(n_f: int, n_t: int) -> int:
    def side(n):
        d = n.bit_length() - 1
        return 2 + sum(2 * l + 4 for l in range(d))
    return 1 + side(n_f) + side(n_t)


def logup_prove(f: np.ndarray, table: np.ndarray, mult: np.ndarray, chal_seed: bytes,
                chal_domain: int):
    f = np.ascontiguousarray(f, dtype=np.int16)
    table = np.ascontiguousarray(table, dtype=np.int16)
    mult = np.ascontiguousarray(mult, dtype=np.uint32)
    cap = logup_prove_words(f.size, table.size)
    out = fp2_array(cap)
    w = lib().or_logup_prove(_p(f), f.size, _p(table), table.size, _p(mult), chal_seed,
                             chal_domain, _p(out), cap)
    assert w == cap, (w, cap)
    return out


def logup_prove_fp(f: np.ndarray, table: np.ndarray, mult: np.ndarray, chal_seed: bytes, chal_domain: int):
    """logup_prove over canonical Fp query and table columns (u64 < p)."""
    f = np.ascontiguousarray(f, dtype=np.uint64)
    table = np.ascontiguousarray(table, dtype=np.uint64)
    mult = np.ascontiguousarray(mult, dtype=np.uint32)
    cap = logup_prove_words(f.size, table.size)
    out = fp2_array(cap)
    w = lib().or_logup_prove_fp(_p(f), f.size, _p(table), table.size, _p(mult), chal_seed,
                                chal_domain & 0xFFFFFFFFFFFFFFFF, _p(out), cap)
    assert w == cap, (w, cap)
    return out


# ---- PCS ------------------------------------------------------------------------

def ntt_batch(msgs: np.ndarray, rows: int, msg_len: int, n: int) -> np.ndarray:
    msgs = np.ascontiguousarray(msgs, dtype=np.uint64)
    out = np.zeros(rows * n, dtype=np.uint64)
    lib().or_ntt_batch(_p(msgs), rows, msg_len, n, _p(out))
    return out


def ntt_fp2_batch(msgs: np.ndarray, rows: int, msg_len: int, n: int) -> np.ndarray:
    msgs = np.ascontiguousarray(msgs, dtype=np.uint64)
    out = fp2_array(rows * n)
    lib().or_ntt_fp2_batch(_p(msgs), rows, msg_len, n, _p(out))
    return out


def blake3(data: bytes) -> bytes:
    buf = np.frombuffer(data, dtype=np.uint8).copy() if data else np.zeros(1, np.uint8)
    out = np.zeros(32, dtype=np.uint8)
    lib().or_blake3(_p(buf), len(data), _p(out))
    return out.tobytes()


def blake3_derive_key(context: str, data: bytes) -> bytes:
    """BLAKE3 derive_key mode (blake3::Hasher::new_derive_key(context))."""
    ctx = context.encode()
    cbuf = np.frombuffer(ctx, dtype=np.uint8).copy() if ctx else np.zeros(1, np.uint8)
    buf = np.frombuffer(data, dtype=np.uint8).copy() if data else np.zeros(1, np.uint8)
    out = np.zeros(32, dtype=np.uint8)
    lib().or_blake3_derive_key(_p(cbuf), len(ctx), _p(buf), len(data), _p(out))
    return out.tobytes()


def hash_fp_columns(m: np.ndarray, rows: int, cols: int) -> np.ndarray:
    m = np.ascontiguousarray(m, dtype=np.uint64)
    out = np.zeros((cols, 32), dtype=np.uint8)
    lib().or_hash_fp_columns(_p(m), rows, cols, _p(out))
    return out


def hash_fp2_columns(m: np.ndarray, rows: int, cols: int) -> np.ndarray:
    m = np.ascontiguousarray(m, dtype=np.uint64)
    out = np.zeros((cols, 32), dtype=np.uint8)
    lib().or_hash_fp2_columns(_p(m), rows, cols, _p(out))
    return out


def merkle_tree(leaves: np.ndarray) -> np.ndarray:
    n = leaves.shape[0]
    tree = np.zeros((2 * n - 1, 32), dtype=np.uint8)
    lib().or_merkle_tree(_p(np.ascontiguousarray(leaves)), n, _p(tree))
    return tree


def merkle_paths(tree: np.ndarray, leaves: int, idx: np.ndarray) -> np.ndarray:
    bits = leaves.bit_length() - 1
    idx = np.ascontiguousarray(idx, dtype=np.uint32)
    out = np.zeros((idx.size * bits, 32), dtype=np.uint8)
    lib().or_merkle_paths(_p(tree), leaves, _p(idx), idx.size, _p(out))
    return out


def pcs_messages(w, pads, rows, cols, pad, code_len):
    out = np.zeros(rows * code_len, dtype=np.uint64)
    lib().or_pcs_messages(_p(w), _p(pads) if pad else None, rows, cols, pad, code_len, _p(out))
    return out


def pcs_combine_rows(w, pads, coeffs, rows, cols, pad, combos):
    out = fp2_array(combos * (cols + pad))
    lib().or_pcs_combine_rows(_p(w), _p(pads) if pad else None, _p(coeffs), rows, cols, pad,
                              combos, _p(out))
    return out


def gemm_i64(a, b, m, k, n):
    out = np.zeros(m * n, dtype=np.int64)
    lib().or_gemm_i64(_p(a), _p(b), _p(out), m, k, n)
    return out


def gemm_requant_auth(a, b, masks, m, k, n, shift):
    out = np.zeros(m * n, dtype=np.int16)
    corr = np.zeros(m * n, dtype=np.uint64)
    lib().or_gemm_requant_auth(_p(a), _p(b), _p(masks), _p(out), _p(corr), m, k, n, shift)
    return out, corr


def fnv_u64(values: np.ndarray, h: int = 0xCBF29CE484222325) -> int:
    v = np.ascontiguousarray(values, dtype=np.uint64).reshape(-1)
    return lib().or_fnv_u64(h, _p(v), v.size)


def ligero_commit_open(row_seed: bytes, rows: int, msg_len: int, code_len: int, queries: int, chal_seed: bytes):
    """Resident Ligero commitment + openings on the CPU
    (rust/volta-pcs/src/ligero.rs:465-505 commit, 1440-1480 openings):
    message row r = FpStream(row_seed, r) x msg_len, zero-padded to code_len,
    forward NTT per row, BLAKE3 column leaves, Merkle tree; query j =
    challenge_fp2().c0 mod code_len from FpStream(chal_seed, u64::MAX).
    Returns (root bytes, indices, columns [queries x rows], paths)."""
    msgs = chacha_fp_rows(row_seed, 0, rows, msg_len)
    code = ntt_batch(msgs, rows, msg_len, code_len).reshape(rows, code_len)
    tree = merkle_tree(hash_fp_columns(code, rows, code_len))
    tx = FpStream(chal_seed, 2**64 - 1)
    idx = np.array([tx.next_fp2()[0] % code_len for _ in range(queries)], dtype=np.uint32)
    cols = np.ascontiguousarray(code[:, idx].T)
    bits = code_len.bit_length() - 1
    paths = merkle_paths(tree, code_len, idx).reshape(queries, bits, 32) if bits else np.zeros((queries, 0, 32), np.uint8)
    return tree[-1].tobytes(), idx, cols, paths


# ---- int16 fixed-point forward primitives (fixed.c) -----------------------------

def _opt(a):
    return _p(a) if a is not None else None


_FIXED_ARGS = {
    "or_fixed_embed": [_vp] * 6 + [_sz] * 5 + [C.c_int32],
    "or_fixed_layer_norm": [_vp] * 11 + [_sz, _sz, C.c_uint32, C.c_uint32],
    "or_fixed_gemm": [_vp] * 8 + [_sz] * 3 + [C.c_uint32],
    "or_fixed_qkv_split": [_vp] * 4 + [_sz] * 2,
    "or_fixed_attention_scores": [_vp] * 5 + [_sz] * 5 + [C.c_uint32],
    "or_fixed_softmax": [_vp] * 9 + [_sz] * 3 + [C.c_uint32] * 3 + [C.c_int],
    "or_fixed_av": [_vp] * 5 + [_sz] * 5 + [C.c_uint32],
    "or_fixed_lookup": [_vp] * 3 + [_sz],
    "or_fixed_requant_i16": [_vp] * 3 + [_sz, C.c_uint32],
    "or_fixed_logits": [_vp] * 3 + [_sz] * 3,
}


def _fx():
    L = lib()
    if not getattr(L, "_fixed_declared", False):
        for name, args in _FIXED_ARGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = None
        L._fixed_declared = True
    return L


def fixed_embed(tokens, wte, wpe, rows, d, vocab, positions, pos0, shift):
    acc = np.zeros(rows * d, np.int64)
    out = np.zeros(rows * d, np.int16)
    err = np.zeros(1, np.uint32)
    _fx().or_fixed_embed(_p(tokens), _p(wte), _p(wpe), _p(acc), _p(out), _p(err), rows, d, vocab, positions, pos0,
                         C.c_int32(shift))
    return acc, out, int(err[0])


def fixed_layer_norm(x, gain, bias, lut, rows, d, var_shift, norm_shift):
    means, vars_, rin = (np.zeros(rows, np.int64) for _ in range(3))
    rout = np.zeros(rows, np.int16)
    acc = np.zeros(rows * d, np.int64)
    out = np.zeros(rows * d, np.int16)
    err = np.zeros(1, np.uint32)
    _fx().or_fixed_layer_norm(_p(x), _p(gain), _p(bias), _p(lut), _p(means), _p(vars_), _p(rin), _p(rout), _p(acc),
                              _p(out), _p(err), rows, d, C.c_uint32(var_shift), C.c_uint32(norm_shift))
    return means, vars_, rin, rout, acc, out, int(err[0])


def fixed_gemm(x, w, bias, residual, m, k, n, shift):
    acc = np.zeros(m * n, np.int64)
    req = np.zeros(m * n, np.int16)
    res_out = np.zeros(m * n, np.int16) if residual is not None else None
    err = np.zeros(1, np.uint32)
    _fx().or_fixed_gemm(_p(x), _p(w), _opt(bias), _opt(residual), _p(acc), _p(req), _opt(res_out), _p(err), m, k, n,
                        C.c_uint32(shift))
    return acc, req, res_out, int(err[0])


def fixed_qkv_split(qkv, rows, d):
    q, k, v = (np.zeros(rows * d, np.int16) for _ in range(3))
    _fx().or_fixed_qkv_split(_p(qkv), _p(q), _p(k), _p(v), rows, d)
    return q, k, v


def packed_len(rows, pos0, heads):
    return heads * (rows * pos0 + rows * (rows + 1) // 2)


def fixed_attention_scores(q, k, rows, seq, pos0, heads, head_dim, shift):
    n = packed_len(rows, pos0, heads)
    acc = np.zeros(n, np.int64)
    out = np.zeros(n, np.int16)
    err = np.zeros(1, np.uint32)
    _fx().or_fixed_attention_scores(_p(q), _p(k), _p(acc), _p(out), _p(err), rows, seq, pos0, heads, head_dim,
                                    C.c_uint32(shift))
    return acc, out, int(err[0])


def fixed_softmax(scores, exp_lut, recip_lut, rows, pos0, heads, recip_den_shift, recip_log2, norm_shift,
                  use_row_shift):
    n = packed_len(rows, pos0, heads)
    row_shifts = np.zeros(heads * rows, np.int16)
    exp_out = np.zeros(n, np.int16)
    denoms = np.zeros(heads * rows, np.int64)
    recips = np.zeros(heads * rows, np.int16)
    weights = np.zeros(n, np.int16)
    err = np.zeros(1, np.uint32)
    _fx().or_fixed_softmax(_p(scores), _p(exp_lut), _p(recip_lut), _p(row_shifts), _p(exp_out), _p(denoms),
                           _p(recips), _p(weights), _p(err), rows, pos0, heads, C.c_uint32(recip_den_shift),
                           C.c_uint32(recip_log2), C.c_uint32(norm_shift), C.c_int(use_row_shift))
    return row_shifts, exp_out, denoms, recips, weights, int(err[0])


def fixed_av(weights, values, rows, seq, pos0, d, heads, shift):
    acc = np.zeros(rows * d, np.int64)
    out = np.zeros(rows * d, np.int16)
    err = np.zeros(1, np.uint32)
    _fx().or_fixed_av(_p(weights), _p(values), _p(acc), _p(out), _p(err), rows, seq, pos0, d, heads,
                      C.c_uint32(shift))
    return acc, out, int(err[0])


def fixed_lookup(x, lut):
    out = np.zeros(x.size, np.int16)
    _fx().or_fixed_lookup(_p(x), _p(lut), _p(out), x.size)
    return out


def fixed_requant_i16(x, shift):
    out = np.zeros(x.size, np.int16)
    err = np.zeros(1, np.uint32)
    _fx().or_fixed_requant_i16(_p(x), _p(out), _p(err), x.size, C.c_uint32(shift))
    return out, int(err[0])


def fixed_logits(x, w, rows, d, vocab):
    out = np.zeros(rows * vocab, np.int64)
    _fx().or_fixed_logits(_p(x), _p(w), _p(out), rows, d, vocab)
    return out


class WiresGeom(C.Structure):
    _fields_ = [(n, C.c_size_t) for n in ("query_rows", "seq", "pos0", "heads", "head_pad", "head_dim", "query_pad",
                                          "seq_pad", "d_pad")] + \
               [(n, C.c_uint32) for n in ("shift_scores", "shift_softmax_norm", "shift_qkv", "recip_den_shift",
                                          "recip_log2")] + \
               [(n, C.c_int32) for n in ("exp_pad_input", "recip_pad_output", "use_row_shift")]


def attention_wires(geom: dict, q, k_cache, own_k, v, scores_acc, scores_q, row_shifts, exp_outputs, denoms, recips,
                    weights, recip_lut, qkv_acc):
    """Attention proof-wire columns (backend.cu:2202-2470): returns
    (rect [9 x entries], rows [13 x head_pad query_pad], above, qkv
    [2 x query_pad 4 d_pad], error)."""
    g = WiresGeom(**geom)
    qr = g.query_rows
    rect = np.zeros(9 * g.head_pad * g.query_pad * g.seq_pad, np.uint64)
    rows = np.zeros(13 * g.head_pad * g.query_pad, np.uint64)
    above = np.zeros(max(1, g.heads * qr * (qr - 1) // 2), np.uint64)
    qkv = np.zeros(2 * g.query_pad * 4 * g.d_pad, np.uint64)
    err = np.zeros(1, np.uint32)
    L = lib()
    L.or_attention_wires.argtypes = [C.POINTER(WiresGeom)] + [_vp] * 18
    L.or_attention_wires.restype = None
    L.or_attention_wires(C.byref(g), *[_p(a) for a in (q, k_cache, own_k, v, scores_acc, scores_q, row_shifts,
                                                       exp_outputs, denoms, recips, weights, recip_lut, qkv_acc,
                                                       rect, rows, above, qkv, err)])
    return rect, rows, above, qkv, int(err[0])
