"""Attention proof wires (volta_cuda_attention_proof_wires_device) against
the oracle on forward tensors built by the oracle itself (so every
consistency check passes), with and without the row-shifted softmax, on a
decode-style band (pos0 > 0), and with a corrupted score accumulator that
must raise the sticky error word."""

import ctypes as C

import numpy as np
import pytest

import fixed_layer as fl

pytestmark = pytest.mark.gpu

_IDS = ["q", "k_cache", "own_k", "v", "scores_acc", "scores_q", "row_shifts", "exp_outputs", "denoms", "recips",
        "softmax_weights", "recip_lut", "qkv_acc", "error", "rect", "rows", "above", "qkv"]


class WiresArgs(C.Structure):
    """include/volta_cuda_backend.h vz_attention_wires_args."""
    _fields_ = [f for n in _IDS for f in ((n + "_id", C.c_uint64), (n + "_offset", C.c_size_t))] + \
               [(n, C.c_size_t) for n in ("query_rows", "seq", "pos0", "heads", "head_pad", "head_dim", "query_pad",
                                          "seq_pad", "d_pad")] + \
               [(n, C.c_uint32) for n in ("shift_scores", "shift_softmax_norm", "shift_qkv", "recip_den_shift",
                                          "recip_log2")] + \
               [(n, C.c_int) for n in ("exp_pad_input", "recip_pad_output", "use_row_shift")]


@pytest.fixture(scope="module")
def be():
    from volta_zk_b200 import accel

    b = accel.CudaBackend(policy=0)
    yield b
    b.close()


def pow2ceil(x):
    return 1 << (x - 1).bit_length()


def make_inputs(oracle, rows, pos0, heads, head_dim, use_row_shift, seed):
    rng = np.random.default_rng(seed)
    seq, d = pos0 + rows, heads * head_dim
    q = rng.integers(-300, 300, size=rows * d).astype(np.int16)
    k_cache = rng.integers(-300, 300, size=seq * d).astype(np.int16)
    own_k = k_cache[pos0 * d:].copy()
    v = rng.integers(-3000, 3000, size=rows * d).astype(np.int16)
    shift_qkv = 10
    out = np.concatenate([q.reshape(rows, d), own_k.reshape(rows, d), v.reshape(rows, d)], axis=1).astype(np.int64)
    qkv_acc = (out << shift_qkv) + rng.integers(0, 1 << shift_qkv, size=out.shape) - (1 << (shift_qkv - 1))
    s_acc, s_q, _ = oracle.fixed_attention_scores(q, k_cache, rows, seq, pos0, heads, head_dim, 10)
    g = np.load(fl.GOLDEN)
    row_shifts, exp_out, denoms, recips, weights, _ = oracle.fixed_softmax(
        s_q, g["exp"], g["softmax_recip"], rows, pos0, heads, 6, 26, 14, use_row_shift)
    geom = dict(query_rows=rows, seq=seq, pos0=pos0, heads=heads, head_pad=pow2ceil(heads), head_dim=head_dim,
                query_pad=pow2ceil(rows), seq_pad=pow2ceil(seq), d_pad=pow2ceil(d), shift_scores=10,
                shift_softmax_norm=14, shift_qkv=shift_qkv, recip_den_shift=6, recip_log2=26, exp_pad_input=-32768,
                recip_pad_output=127, use_row_shift=use_row_shift)
    arrays = dict(q=q, k_cache=k_cache, own_k=own_k, v=v, scores_acc=s_acc, scores_q=s_q, row_shifts=row_shifts,
                  exp_outputs=exp_out, denoms=denoms, recips=recips, softmax_weights=weights,
                  recip_lut=g["softmax_recip"], qkv_acc=np.ascontiguousarray(qkv_acc.reshape(-1)))
    return geom, arrays


def run_device(be, geom, arrays):
    qr = geom["query_rows"]
    sizes = dict(rect=9 * geom["head_pad"] * geom["query_pad"] * geom["seq_pad"],
                 rows=13 * geom["head_pad"] * geom["query_pad"],
                 above=max(1, geom["heads"] * qr * (qr - 1) // 2),
                 qkv=2 * geom["query_pad"] * 4 * geom["d_pad"])
    a = WiresArgs(**geom)
    ids = []
    for name, arr in arrays.items():
        i = be.upload_new(arr)
        ids.append(i)
        setattr(a, name + "_id", i)
    err = be.upload_new(np.zeros(1, np.uint32))
    a.error_id = err
    outs = {}
    for name, n in sizes.items():
        outs[name] = be.alloc(8 * n)
        setattr(a, name + "_id", outs[name])
    rc = be.lib.volta_cuda_attention_proof_wires_device(be.ctx, C.byref(a))
    assert rc == 0, be.last_error()
    res = [be.download(outs[n], 8 * sizes[n]) for n in ("rect", "rows", "above", "qkv")]
    res.append(int(be.download(err, 4, dtype=np.uint32)[0]))
    for i in ids + [err] + list(outs.values()):
        be.free(i)
    return res


def oracle_wires(oracle, geom, arrays):
    x = arrays
    return oracle.attention_wires(geom, x["q"], x["k_cache"], x["own_k"], x["v"], x["scores_acc"], x["scores_q"],
                                  x["row_shifts"], x["exp_outputs"], x["denoms"], x["recips"], x["softmax_weights"],
                                  x["recip_lut"], x["qkv_acc"])


@pytest.mark.parametrize("rows,pos0,heads,head_dim", [(2, 0, 1, 8), (5, 3, 2, 16), (16, 0, 12, 64), (7, 20, 3, 32)])
@pytest.mark.parametrize("use_row_shift", [0, 1])
def test_wires_match_oracle(be, oracle, rows, pos0, heads, head_dim, use_row_shift):
    geom, arrays = make_inputs(oracle, rows, pos0, heads, head_dim, use_row_shift, rows * 31 + pos0)
    exp = oracle_wires(oracle, geom, arrays)
    got = run_device(be, geom, arrays)
    for k, (g, e) in enumerate(zip(got[:4], exp[:4])):
        assert np.array_equal(g, e), k
    assert got[4] == exp[4]


def test_wires_flag_inconsistent_scores(be, oracle):
    geom, arrays = make_inputs(oracle, 5, 3, 2, 16, 1, 99)
    arrays["scores_acc"] = arrays["scores_acc"].copy()
    arrays["scores_acc"][4] += 1
    exp = oracle_wires(oracle, geom, arrays)
    got = run_device(be, geom, arrays)
    assert exp[4] == 1 and got[4] == 1
    assert all(np.array_equal(g, e) for g, e in zip(got[:4], exp[:4]))


def test_wires_reject_bad_geometry(be, oracle):
    geom, arrays = make_inputs(oracle, 5, 3, 2, 16, 0, 7)
    a = WiresArgs(**dict(geom, query_rows=1))
    assert be.lib.volta_cuda_attention_proof_wires_device(be.ctx, C.byref(a)) != 0
    a = WiresArgs(**dict(geom, seq_pad=12))
    assert be.lib.volta_cuda_attention_proof_wires_device(be.ctx, C.byref(a)) != 0
