"""Shared driver for the fixed-point layer parity tests: regenerates the
synthetic layer (rust/volta-gpt2/src/layer.rs synthetic_weights /
synthetic_input: one splitmix64 stream) and binds the device's seam
primitives (DeviceOps) for the oracle's forward_layer composition
(oracle/gpt2.py, restating scripts/gpt2_fixed.py forward_layer), which
returns every intermediate."""

import hashlib
import os

import numpy as np

from oracle.gpt2 import OracleOps, forward_layer, forward_model  # noqa: F401  (the oracle's compositions)

D, H, DH, DFF = 768, 12, 64, 3072
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "fixed_layer_t8.npz")
# P4 LutParams defaults (gpt2_fixed.py LutParams / luts.rs)
LN_VAR_SHIFT, SHIFT_LN_NORM, RECIP_DEN_SHIFT, RECIP_LOG2 = 7, 16, 6, 26
SHIFT_QKV, SHIFT_SCORES, SHIFT_SOFTMAX_NORM, SHIFT_AV = 10, 10, 14, 12
SHIFT_ATTN_PROJ, SHIFT_FFN_UP, SHIFT_FFN_DOWN = 10, 10, 10

_M = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64_stream(seed: int, n: int, start: int = 0) -> np.ndarray:
    """Outputs start..start+n of splitmix64 (state += 0x9E3779B97F4A7C15,
    then the xor-shift-multiply finaliser), vectorised."""
    with np.errstate(over="ignore"):
        idx = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        z = np.uint64(seed) + idx * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def synthetic_layer(seed: int, t: int):
    sizes = [D * 3 * D, D * D, D * DFF, DFF * D]
    pos = 0
    mats = []
    for n in sizes:
        mats.append(((splitmix64_stream(seed, n, pos) % np.uint64(127)).astype(np.int64) - 63).astype(np.int16))
        pos += n
    gains = []
    for _ in range(2):
        gains.append((48 + (splitmix64_stream(seed, D, pos) % np.uint64(33)).astype(np.int64)).astype(np.int16))
        pos += D
    biases = []
    for _ in range(2):
        biases.append(((splitmix64_stream(seed, D, pos) % np.uint64(256)).astype(np.int64) - 128).astype(np.int16))
        pos += D
    x = ((splitmix64_stream(seed ^ 0xA5A5A5A5A5A5A5A5, t * D) % np.uint64(2048)).astype(np.int64) - 1024)
    w = dict(c_attn=mats[0], attn_proj=mats[1], ffn_up=mats[2], ffn_down=mats[3], ln1_gain=gains[0],
             ln2_gain=gains[1], ln1_bias=biases[0], ln2_bias=biases[1])
    return w, x.astype(np.int16)


def weights_digest(w) -> str:
    cat = np.concatenate([w["c_attn"], w["attn_proj"], w["ffn_up"], w["ffn_down"], w["ln1_gain"], w["ln1_bias"],
                          w["ln2_gain"], w["ln2_bias"]])
    return hashlib.sha256(cat.tobytes()).hexdigest()


def digest(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def check_against_golden(result):
    """(name, expected dtype) pairs whose digests differ from the fixture."""
    g = np.load(GOLDEN)
    bad = []
    for key in [k[4:] for k in g.files if k.startswith("sha_")]:
        arr = np.ascontiguousarray(result[key]).astype(str(g["dtype_" + key]))
        # the reference keeps denoms/recips as (H, t) and the accumulators as
        # 2-D arrays: digests are over the row-major bytes, so flat == 2-D
        if digest(arr) != str(g["sha_" + key]):
            bad.append(key)
    return bad


class DeviceOps:
    """The same primitives through the seam's resident entry points
    (volta_cuda_fixed_*_device) of a CudaBackend; each call uploads its
    inputs, runs the device kernel and downloads every output."""

    def __init__(self, be):
        self.be = be

    def _err(self):
        return self.be.upload_new(np.zeros(1, np.uint32))

    def _get(self, buf, n, dtype):
        return self.be.download(buf, n * np.dtype(dtype).itemsize, dtype=dtype)

    def _free(self, *ids):
        for i in ids:
            if i:
                self.be.free(i)

    def layer_norm(self, x, gain, bias, lut, rows, d, var_shift, norm_shift):
        be = self.be
        ins = [be.upload_new(a) for a in (x, gain, bias, lut)]
        outs = [be.alloc(8 * rows) for _ in range(3)] + [be.alloc(2 * rows), be.alloc(8 * rows * d),
                                                        be.alloc(2 * rows * d)]
        err = self._err()
        be.call("fixed_layer_norm_device", ins[0], 0, ins[1], 0, ins[2], 0, ins[3], 0, outs[0], 0, outs[1], 0,
                outs[2], 0, outs[3], 0, outs[4], 0, outs[5], 0, err, 0, rows, d, var_shift, norm_shift)
        res = (self._get(outs[0], rows, np.int64), self._get(outs[1], rows, np.int64),
               self._get(outs[2], rows, np.int64), self._get(outs[3], rows, np.int16),
               self._get(outs[4], rows * d, np.int64), self._get(outs[5], rows * d, np.int16),
               int(self._get(err, 1, np.uint32)[0]))
        self._free(*ins, *outs, err)
        return res

    def gemm(self, x, w, bias, residual, m, k, n, shift):
        be = self.be
        xi, wi = be.upload_new(x), be.upload_new(w)
        bi = be.upload_new(bias) if bias is not None else 0
        ri = be.upload_new(residual) if residual is not None else 0
        acc, req = be.alloc(8 * m * n), be.alloc(2 * m * n)
        ro = be.alloc(2 * m * n) if residual is not None else 0
        err = self._err()
        be.call("fixed_gemm_device", xi, 0, wi, 0, bi, 0, ri, 0, acc, 0, req, 0, ro, 0, err, 0, m, k, n, shift)
        res = (self._get(acc, m * n, np.int64), self._get(req, m * n, np.int16),
               self._get(ro, m * n, np.int16) if ro else None, int(self._get(err, 1, np.uint32)[0]))
        self._free(xi, wi, bi, ri, acc, req, ro, err)
        return res

    def qkv_split(self, qkv, rows, d):
        be = self.be
        src = be.upload_new(qkv)
        outs = [be.alloc(2 * rows * d) for _ in range(3)]
        be.call("fixed_qkv_split_device", src, 0, outs[0], 0, outs[1], 0, outs[2], 0, rows, d)
        res = tuple(self._get(o, rows * d, np.int16) for o in outs)
        self._free(src, *outs)
        return res

    def scores(self, q, k, rows, seq, pos0, heads, head_dim, shift):
        be = self.be
        n = heads * (rows * pos0 + rows * (rows + 1) // 2)
        qi, ki = be.upload_new(q), be.upload_new(k)
        acc, out, err = be.alloc(8 * n), be.alloc(2 * n), self._err()
        be.call("fixed_attention_scores_device", qi, 0, ki, 0, acc, 0, out, 0, err, 0, rows, seq, pos0, heads,
                head_dim, shift)
        res = (self._get(acc, n, np.int64), self._get(out, n, np.int16), int(self._get(err, 1, np.uint32)[0]))
        self._free(qi, ki, acc, out, err)
        return res

    def softmax(self, scores, exp_lut, recip_lut, rows, pos0, heads, den_shift, recip_log2, norm_shift, row_shift):
        be = self.be
        n = heads * (rows * pos0 + rows * (rows + 1) // 2)
        rc = heads * rows
        ins = [be.upload_new(a) for a in (scores, exp_lut, recip_lut)]
        rs, ex, dn, rp, wt = be.alloc(2 * rc), be.alloc(2 * n), be.alloc(8 * rc), be.alloc(2 * rc), be.alloc(2 * n)
        err = self._err()
        be.call("fixed_softmax_device", ins[0], 0, ins[1], 0, ins[2], 0, rs, 0, ex, 0, dn, 0, rp, 0, wt, 0, err, 0,
                rows, pos0 + rows, pos0, heads, den_shift, recip_log2, norm_shift, row_shift)
        res = (self._get(rs, rc, np.int16), self._get(ex, n, np.int16), self._get(dn, rc, np.int64),
               self._get(rp, rc, np.int16), self._get(wt, n, np.int16), int(self._get(err, 1, np.uint32)[0]))
        self._free(*ins, rs, ex, dn, rp, wt, err)
        return res

    def av(self, weights, values, rows, seq, pos0, d, heads, shift):
        be = self.be
        wi, vi = be.upload_new(weights), be.upload_new(values)
        acc, out, err = be.alloc(8 * rows * d), be.alloc(2 * rows * d), self._err()
        be.call("fixed_av_device", wi, 0, vi, 0, acc, 0, out, 0, err, 0, rows, seq, pos0, d, heads, shift)
        res = (self._get(acc, rows * d, np.int64), self._get(out, rows * d, np.int16),
               int(self._get(err, 1, np.uint32)[0]))
        self._free(wi, vi, acc, out, err)
        return res

    def lookup(self, x, lut):
        be = self.be
        xi, li, out = be.upload_new(x), be.upload_new(lut), be.alloc(2 * x.size)
        be.call("fixed_lookup_device", xi, 0, li, 0, out, 0, x.size)
        res = self._get(out, x.size, np.int16)
        self._free(xi, li, out)
        return res
