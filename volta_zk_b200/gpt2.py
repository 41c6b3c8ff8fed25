"""GPT-2 small int16 fixed-point model: synthetic weights, lookup tables and
the whole-model device session (config 3's witness forward).

Input synthesis restates the reference's generators:
  * synthetic_model (rust/volta-gpt2/src/model.rs:504-600): layer l's weights
    from synthetic_weights_for_config(seed + l * 0x9E3779B9)
    (layer.rs:283-309, one splitmix64 stream per layer: c_attn, attn_proj,
    ffn_up, ffn_down, ln1/ln2 gains, ln1/ln2 biases), zero GEMM biases, wte
    then wpe from one LCG, final LN gain 64 / bias 0, tied output;
  * build_luts (rust/volta-gpt2/src/luts.rs:133-173, mirrored by
    scripts/gpt2_fixed.py:112-166): the exp, gelu, ln_rsqrt and
    softmax_recip tables, f64 math with round-half-away-from-zero.
The session runs the forward on the device (libvolta_accel.so
vzh_gpt2_*, over the seam's volta_cuda_fixed_*_device entry points).
"""

from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field

import numpy as np

VOCAB, POSITIONS, D, HEADS, HEAD_DIM, DFF, LAYERS = 50257, 1024, 768, 12, 64, 3072, 12
TOKEN_SEED = bytes([0x70] * 32)
MODEL_SEED = 0x1234
TABLE_LEN = 1 << 16
I16_MIN, I16_MAX = -32768, 32767


@dataclass
class LutParams:
    """luts.rs LutParams::default, with the P5 stable softmax switch."""
    ln_var_shift: int = 7
    ln_rsqrt_log2: int = 18
    shift_ln_norm: int = 16
    exp_in_log2: int = 10
    exp_out_log2: int = 12
    recip_den_shift: int = 6
    recip_log2: int = 26
    gelu_scale_log2: int = 10
    shift_qkv: int = 10
    shift_scores: int = 10
    shift_softmax_norm: int = 14
    shift_av: int = 12
    shift_attn_proj: int = 10
    shift_ffn_up: int = 10
    shift_ffn_down: int = 10
    softmax_row_shift: bool = True
    shift_embed: int = 0


def _round_away(v: float) -> int:
    """f64::round (half away from zero)."""
    return math.floor(v + 0.5) if v >= 0 else math.ceil(v - 0.5)


def build_luts(p: LutParams | None = None) -> dict:
    """The four int16 tables of luts.rs build_luts (65536 entries each; exp
    and gelu indexed by the i16 input's u16 bit pattern)."""
    p = p or LutParams()
    exp_in, exp_out, gelu_s = float(1 << p.exp_in_log2), float(1 << p.exp_out_log2), float(1 << p.gelu_scale_log2)
    exp_tab = np.zeros(TABLE_LEN, dtype=np.int16)
    gelu_tab = np.zeros(TABLE_LEN, dtype=np.int16)
    rsqrt_tab = np.zeros(TABLE_LEN, dtype=np.int16)
    recip_tab = np.zeros(TABLE_LEN, dtype=np.int16)
    for u in range(TABLE_LEN):
        x = u - 65536 if u >= 32768 else u
        exp_tab[u] = min(_round_away(exp_out * (2.0 ** (x / exp_in))), I16_MAX)
        xr = x / gelu_s
        g = 0.5 * xr * (1.0 + math.tanh(0.7978845608028654 * (xr + 0.044715 * xr * xr * xr)))
        gelu_tab[u] = max(I16_MIN, min(I16_MAX, _round_away(g * gelu_s)))
        s = math.isqrt((u + 1) << p.ln_var_shift)
        rsqrt_tab[u] = min(((1 << p.ln_rsqrt_log2) + s // 2) // s, I16_MAX)
        den = (u << p.recip_den_shift) + (1 << (p.recip_den_shift - 1))
        recip_tab[u] = min(((1 << p.recip_log2) + den // 2) // den, I16_MAX)
    return {"exp": exp_tab, "gelu": gelu_tab, "ln_rsqrt": rsqrt_tab, "softmax_recip": recip_tab}


_U64 = np.uint64


def splitmix64_stream(seed: int, n: int, start: int = 0) -> np.ndarray:
    """Outputs start..start+n of splitmix64 from `seed` (state +=
    0x9E3779B97F4A7C15, then the xor-shift-multiply finaliser), vectorised."""
    with np.errstate(over="ignore"):
        idx = np.arange(start + 1, start + n + 1, dtype=_U64)
        z = _U64(seed & 0xFFFFFFFFFFFFFFFF) + idx * _U64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> _U64(30))) * _U64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> _U64(27))) * _U64(0x94D049BB133111EB)
        return z ^ (z >> _U64(31))


def lcg_values(state: int, n: int, radius: int):
    """n draws of x <- x * 6364136223846793005 + 1442695040888963407 (mod 2^64)
    mapped to x mod (2r+1) - r; returns (values, state after the last draw).
    Vectorised through the closed form x_k = a^k x_0 + c (1 + a + ... +
    a^(k-1)), whose powers and sums numpy accumulates mod 2^64."""
    a, c = _U64(6364136223846793005), _U64(1442695040888963407)
    with np.errstate(over="ignore"):
        ak = np.cumprod(np.full(n, a, dtype=_U64), dtype=_U64)       # a^1 .. a^n
        geo = np.empty(n, dtype=_U64)                                 # 1 + a + ... + a^(k-1)
        geo[0] = _U64(1)
        if n > 1:
            geo[1:] = ak[:-1]
        geo = np.cumsum(geo, dtype=_U64)
        x = ak * _U64(state & 0xFFFFFFFFFFFFFFFF) + c * geo
    vals = (x % _U64(2 * radius + 1)).astype(np.int64) - radius
    return vals.astype(np.int16), int(x[-1])


@dataclass
class Gpt2Model:
    layers: list = field(default_factory=list)   # dicts of int16 arrays (k x n GEMM weights)
    wte: np.ndarray = None
    wpe: np.ndarray = None
    lnf_gain: np.ndarray = None
    lnf_bias: np.ndarray = None

    @property
    def shape(self) -> "Gpt2Shape":
        """The shape the weights carry (heads of 64)."""
        vocab, d = self.wte.shape
        return Gpt2Shape(layers=len(self.layers), d=d, heads=d // HEAD_DIM, head_dim=HEAD_DIM,
                         dff=self.layers[0]["ffn_up"].shape[1], vocab=vocab, positions=self.wpe.shape[0])


@dataclass(frozen=True)
class Gpt2Shape:
    """A dense GPT-2 shape (ModelConfig's fields for a full-causal
    LayerNorm/GELU model with n_kv_heads = n_q_heads, model.rs)."""
    layers: int = LAYERS
    d: int = D
    heads: int = HEADS
    head_dim: int = HEAD_DIM
    dff: int = DFF
    vocab: int = VOCAB
    positions: int = POSITIONS


GPT2_SMALL = Gpt2Shape()
# The scaled synthetic shape of the decode/scaling configuration: 24 layers,
# d_model 1024, 16 heads of 64, MLP 4096 (a ModelConfig with the GPT-2 small
# vocabulary and context), proved at 512 tokens.
GPT2_SCALED = Gpt2Shape(layers=24, d=1024, heads=16, dff=4096)


def synthetic_layer_weights(seed: int, d: int = D, dff: int = DFF) -> dict:
    """layer.rs synthetic_weights_for_config (283-309) for a dense shape
    (qkv_dim = 3 d)."""
    D, DFF = d, dff
    sizes = [D * 3 * D, D * D, D * DFF, DFF * D]
    shapes = [(D, 3 * D), (D, D), (D, DFF), (DFF, D)]
    pos, mats = 0, []
    for n, shp in zip(sizes, shapes):
        mats.append(((splitmix64_stream(seed, n, pos) % _U64(127)).astype(np.int64) - 63).astype(np.int16)
                    .reshape(shp))
        pos += n
    vec = []
    for mod, off in ((33, 48), (33, 48), (256, -128), (256, -128)):
        vec.append(((splitmix64_stream(seed, D, pos) % _U64(mod)).astype(np.int64) + off).astype(np.int16))
        pos += D
    return dict(c_attn=mats[0], attn_proj=mats[1], ffn_up=mats[2], ffn_down=mats[3], ln1_gain=vec[0],
                ln2_gain=vec[1], ln1_bias=vec[2], ln2_bias=vec[3])


def synthetic_model(seed: int = MODEL_SEED, n_layers: int | None = None, shape: Gpt2Shape = GPT2_SMALL) -> Gpt2Model:
    """model.rs synthetic_model (504-585): per-layer synthetic weights at
    seed + layer * 0x9E3779B9, zero GEMM biases, then wte (radius 15), wpe
    (radius 7) from one LCG, final LN gain 64 and bias 0.  n_layers
    overrides shape.layers (a model cut short for tests)."""
    n_layers = shape.layers if n_layers is None else n_layers
    D, VOCAB, POSITIONS = shape.d, shape.vocab, shape.positions
    layers = [synthetic_layer_weights((seed + l * 0x9E3779B9) & 0xFFFFFFFFFFFFFFFF, D, shape.dff)
              for l in range(n_layers)]
    wte, state = lcg_values(seed ^ 0xD1B54A32D192ED03, VOCAB * D, 15)
    wpe, _ = lcg_values(state, POSITIONS * D, 7)
    return Gpt2Model(layers=layers, wte=wte.reshape(VOCAB, D), wpe=wpe.reshape(POSITIONS, D),
                     lnf_gain=np.full(D, 64, dtype=np.int16), lnf_bias=np.zeros(D, dtype=np.int16))


def prefill_tokens(t: int) -> np.ndarray:
    """FpStream::domain_separated([0x70; 32], 0).next_fp() mod 50257, t ids (u32)."""
    from .accel import fpstream_fp_rows

    return (fpstream_fp_rows(TOKEN_SEED, 0, t) % _U64(VOCAB)).astype(np.uint32)


# Proof sites of one layer in word order (host/gpt2.hpp Gpt2Site): the 14
# lookup instances, then the GEMM, attention and LayerNorm sumchecks; site 0
# (the VOLE-MAC boundary corrections) has no words.  A unit's mask has bit k
# for site k.
SITE_ORDER = list(range(1, 15)) + list(range(16, 25))
SITE_CORRECTIONS = 0
ALL_SITES = 0x1FF7FFF
# The two parts a layer's proof splits into when a GPU split needs finer
# units: the attention-rectangle sites (the three 16 x T_pad^2 lookups, the
# reciprocal lookup and the A.V, softmax-norm and Q.K^T sumchecks) and the
# rest.  Their device times at T = 1024 on a B200 (ms, in a sequence of
# 12): a whole layer 10.9, the parts 6.55 and 4.4, the weight commitment 6.8.
PART_ATTENTION = sum(1 << k for k in (8, 9, 10, 11, 20, 21, 22))
PART_REST = ALL_SITES & ~PART_ATTENTION
LAYER_COST, PART_COSTS, COMMIT_COST = 10.9, {PART_ATTENTION: 6.55, PART_REST: 4.4}, 6.8
# The same costs for the scaled shape (GPT2_SCALED) at T = 512, measured the
# same way (24 in a row): a layer 6.06, its parts 2.63 and 3.49, the 2^15-row
# weight commitment 27.55 (ms on a B200).
SCALED_COSTS = (6.06, {PART_ATTENTION: 2.63, PART_REST: 3.49}, 27.55)

# wire names, in the order of gpt2.hpp's Gpt2Wire
WIRES = ["x_in", "ln1_mean", "ln1_var", "ln1_rsqrt_in", "ln1_rsqrt_out", "ln1_acc", "ln1_out", "qkv_acc", "qkv_q",
         "q", "k", "v", "scores_acc", "scores_q", "row_shift", "exp_out", "denoms", "recips", "weights", "av_acc",
         "av_q", "proj_acc", "attn_proj_q", "attn_block_out", "ln2_mean", "ln2_var", "ln2_rsqrt_in", "ln2_rsqrt_out",
         "ln2_acc", "ln2_out", "ffn_up_acc", "ffn_up_q", "gelu_out", "ffn_down_acc", "ffn_down_q", "ffn_block_out",
         "error"]


def wire_dtype_count(name: str, t: int, shape: "Gpt2Shape" = None):
    shape = shape or GPT2_SMALL
    D, HEADS, DFF = shape.d, shape.heads, shape.dff
    td, n, ht = t * D, HEADS * (t * (t + 1) // 2), HEADS * t
    i16, i64 = np.int16, np.int64
    table = {"ln1_mean": (i64, t), "ln1_var": (i64, t), "ln1_rsqrt_in": (i64, t), "ln1_rsqrt_out": (i16, t),
             "ln2_mean": (i64, t), "ln2_var": (i64, t), "ln2_rsqrt_in": (i64, t), "ln2_rsqrt_out": (i16, t),
             "ln1_acc": (i64, td), "ln2_acc": (i64, td), "av_acc": (i64, td), "proj_acc": (i64, td),
             "ffn_down_acc": (i64, td), "qkv_acc": (i64, 3 * td), "qkv_q": (i16, 3 * td), "scores_acc": (i64, n),
             "scores_q": (i16, n), "exp_out": (i16, n), "weights": (i16, n), "row_shift": (i16, ht),
             "recips": (i16, ht), "denoms": (i64, ht), "ffn_up_acc": (i64, t * DFF), "ffn_up_q": (i16, t * DFF),
             "gelu_out": (i16, t * DFF), "error": (np.uint32, 1)}
    return table.get(name, (i16, td))


class Gpt2Session:
    """The whole model resident on one device context (weights uploaded
    once); forward() enqueues embed -> 12 layers -> final LN -> logits."""

    def __init__(self, prover, model: Gpt2Model, t: int, luts: dict | None = None, params: LutParams | None = None):
        from . import accel

        self.prover, self.be, self.t = prover, prover.backend, t
        self.params = params or LutParams()
        self.luts = luts or build_luts(self.params)
        self.host = accel.load_host_library()
        L = self.host
        L.vzh_gpt2_open.restype = C.c_void_p
        L.vzh_gpt2_open.argtypes = [C.c_void_p] * 10 + [C.c_char_p, C.c_size_t]
        L.vzh_gpt2_close.argtypes = [C.c_void_p]
        L.vzh_gpt2_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        L.vzh_gpt2_buffer.restype = C.c_uint64
        L.vzh_gpt2_buffer.argtypes = [C.c_void_p, C.c_size_t, C.c_int]
        p = self.params
        self._keep = []
        self.shape = sh = model.shape
        dims = np.array([sh.layers, sh.d, sh.heads, sh.head_dim, sh.dff, sh.vocab, sh.positions, t], dtype=np.uint64)
        shifts = np.array([p.ln_var_shift, p.shift_ln_norm, p.recip_den_shift, p.recip_log2, p.shift_qkv,
                           p.shift_scores, p.shift_softmax_norm, p.shift_av, p.shift_attn_proj, p.shift_ffn_up,
                           p.shift_ffn_down, p.shift_embed & 0xFFFFFFFF, int(p.softmax_row_shift)], dtype=np.uint32)
        ptrs = []
        for lw in model.layers:
            for k in ("c_attn", "attn_proj", "ffn_up", "ffn_down", "ln1_gain", "ln1_bias", "ln2_gain", "ln2_bias"):
                a = np.ascontiguousarray(lw[k], dtype=np.int16)
                self._keep.append(a)
                ptrs.append(a.ctypes.data)
        wptr = (C.c_void_p * len(ptrs))(*ptrs)
        lut_arrays = [np.ascontiguousarray(self.luts[k], dtype=np.int16)
                      for k in ("ln_rsqrt", "exp", "softmax_recip", "gelu")]
        lptr = (C.c_void_p * 4)(*[a.ctypes.data for a in lut_arrays])
        llen = np.array([a.size for a in lut_arrays], dtype=np.uint64)
        host = [np.ascontiguousarray(x, dtype=np.int16) for x in (model.wte, model.wpe, model.lnf_gain, model.lnf_bias)]
        err = C.create_string_buffer(1024)
        self.h = L.vzh_gpt2_open(prover.h, dims.ctypes.data, shifts.ctypes.data, C.cast(wptr, C.c_void_p),
                                 *[x.ctypes.data for x in host], C.cast(lptr, C.c_void_p), llen.ctypes.data, err, 1024)
        if not self.h:
            raise accel.AccelError(err.value.decode())

    def close(self):
        if self.h:
            self.host.vzh_gpt2_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def forward(self, tokens: np.ndarray | None = None):
        """Enqueue the forward (tokens: t u32 ids from host memory, else the
        resident token buffer); nothing is downloaded."""
        from . import accel

        err = C.create_string_buffer(1024)
        ptr = None
        if tokens is not None:
            tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
            assert tokens.size == self.t
            ptr = tokens.ctypes.data
        if self.host.vzh_gpt2_forward(self.h, ptr, err, 1024) != 0:
            raise accel.AccelError(err.value.decode())

    def buffer(self, layer, which: int) -> int:
        return int(self.host.vzh_gpt2_buffer(self.h, C.c_size_t(layer if layer is not None else 2**64 - 1), which))

    def wire(self, layer: int, name: str) -> np.ndarray:
        dtype, count = wire_dtype_count(name, self.t, self.shape)
        return self.be.download(self.buffer(layer, WIRES.index(name)), count * np.dtype(dtype).itemsize, dtype=dtype)

    def logits(self) -> np.ndarray:
        return self.be.download(self.buffer(None, 2), self.shape.vocab * 8, dtype=np.int64)

    def embed_out(self) -> np.ndarray:
        return self.wire(0, "x_in")

    def final_ln_out(self) -> np.ndarray:
        return self.be.download(self.buffer(None, 9), self.shape.d * 2, dtype=np.int16)

    def error_word(self) -> int:
        return int(self.be.download(self.buffer(None, 3), 4, dtype=np.uint32)[0])

    def layer_errors(self):
        return [int(self.wire(l, "error")[0]) for l in range(self.shape.layers)]

    def band(self, t0: int) -> "Gpt2Band":
        """The band witness of rows t0 .. t-1 of the last forward (built)."""
        return Gpt2Band(self, t0)

    def decoder(self, max_steps: int = 0) -> "Gpt2Decoder":
        """KV-cached greedy decoding after the last forward (at most max_steps
        steps; 0: up to the last position)."""
        return Gpt2Decoder(self, max_steps)


def _bind_decode(L):
    vp, sz, u64 = C.c_void_p, C.c_size_t, C.c_uint64
    L.vzh_gpt2_band_open.restype = vp
    L.vzh_gpt2_band_open.argtypes = [vp, sz, C.c_char_p, sz]
    L.vzh_gpt2_band_close.argtypes = [vp]
    L.vzh_gpt2_band_build.argtypes = [vp, C.c_char_p, sz]
    L.vzh_gpt2_band_buffer.argtypes = [vp, sz, C.c_int, C.POINTER(u64), C.POINTER(sz), C.c_char_p, sz]
    L.vzh_gpt2_decoder_open.restype = vp
    L.vzh_gpt2_decoder_open.argtypes = [vp, sz, C.c_char_p, sz]
    L.vzh_gpt2_decoder_close.argtypes = [vp]
    L.vzh_gpt2_decode.argtypes = [vp, sz, C.c_char_p, sz]
    L.vzh_gpt2_decoder_buffer.restype = u64
    L.vzh_gpt2_decoder_buffer.argtypes = [vp, sz, C.c_int]


def band_dtype_count(name: str, t0: int, q: int, shape: "Gpt2Shape" = None):
    """Element type and count of a band wire (band.rs:112-150 layouts)."""
    shape = shape or GPT2_SMALL
    HEADS = shape.heads
    bc = HEADS * (q * t0 + q * (q + 1) // 2)
    packed = {"scores_acc": np.int64, "scores_q": np.int16, "exp_out": np.int16, "weights": np.int16}
    tables = {"row_shift": np.int16, "denoms": np.int64, "recips": np.int16}
    if name in packed:
        return packed[name], bc
    if name in tables:
        return tables[name], HEADS * q
    return wire_dtype_count(name, q, shape)


class Gpt2Band:
    """Band witness (rust/volta-gpt2/src/band.rs:77-196): rows t0 .. t-1 of a
    session's forward, the per-head packed wires in band packing, the final
    LayerNorm and the logits of every band row."""

    def __init__(self, session: Gpt2Session, t0: int):
        from . import accel

        self.s, self.t0, self.q = session, t0, session.t - t0
        self.L = session.host
        _bind_decode(self.L)
        err = C.create_string_buffer(1024)
        self.h = self.L.vzh_gpt2_band_open(session.h, t0, err, 1024)
        if not self.h:
            raise accel.AccelError(err.value.decode())
        self._check(self.L.vzh_gpt2_band_build(self.h, err, 1024), err)

    @staticmethod
    def _check(rc, err):
        from . import accel

        if rc != 0:
            raise accel.AccelError(err.value.decode())

    def close(self):
        if self.h:
            self.L.vzh_gpt2_band_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _buffer(self, layer, which):
        bid, off = C.c_uint64(), C.c_size_t()
        err = C.create_string_buffer(1024)
        self._check(self.L.vzh_gpt2_band_buffer(self.h, C.c_size_t(layer if layer is not None else 2**64 - 1), which,
                                                C.byref(bid), C.byref(off), err, 1024), err)
        return bid.value, off.value

    def wire(self, layer: int, name: str) -> np.ndarray:
        dtype, count = band_dtype_count(name, self.t0, self.q, self.s.shape)
        bid, off = self._buffer(layer, WIRES.index(name))
        size = np.dtype(dtype).itemsize
        return self.s.be.download(bid, count * size, dtype=dtype, offset_bytes=off * size)

    def final_ln(self, which: int) -> np.ndarray:
        """0 mean, 1 var, 2 rsqrt input, 3 rsqrt output, 4 acc, 5 out, over the q rows."""
        q, qd = self.q, self.q * self.s.shape.d
        dt, n = [(np.int64, q), (np.int64, q), (np.int64, q), (np.int16, q), (np.int64, qd), (np.int16, qd)][which]
        bid, _ = self._buffer(None, which)
        return self.s.be.download(bid, n * np.dtype(dt).itemsize, dtype=dt)

    def logits(self) -> np.ndarray:
        bid, _ = self._buffer(None, 6)
        vocab = self.s.shape.vocab
        return self.s.be.download(bid, self.q * vocab * 8, dtype=np.int64).reshape(self.q, vocab)

    def error_word(self) -> int:
        bid, _ = self._buffer(None, 7)
        return int(self.s.be.download(bid, 4, dtype=np.uint32)[0])


class Gpt2Decoder:
    """KV-cached greedy decoding (rust/volta-gpt2/src/decode.rs:80-300) on
    the device: the caches start from the session's K/V rows, every step runs
    the model on one new row and picks the next token on the device."""

    def __init__(self, session: Gpt2Session, max_steps: int = 0):
        from . import accel

        self.s = session
        self.L = session.host
        _bind_decode(self.L)
        err = C.create_string_buffer(1024)
        self.h = self.L.vzh_gpt2_decoder_open(session.h, max_steps, err, 1024)
        if not self.h:
            raise accel.AccelError(err.value.decode())
        self.generated = 0

    def close(self):
        if self.h:
            self.L.vzh_gpt2_decoder_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def generate(self, n: int):
        """Enqueue n more greedy steps (nothing is downloaded)."""
        from . import accel

        err = C.create_string_buffer(1024)
        if self.L.vzh_gpt2_decode(self.h, n, err, 1024) != 0:
            raise accel.AccelError(err.value.decode())
        self.generated += n

    def tokens(self) -> np.ndarray:
        """The generated tokens so far (token i was fed to step i)."""
        buf = int(self.L.vzh_gpt2_decoder_buffer(self.h, 0, 0))
        return self.s.be.download(buf, 4 * self.generated, dtype=np.uint32)

    def logits(self) -> np.ndarray:
        """Step i's logits row (the row that sampled token i + 1)."""
        buf = int(self.L.vzh_gpt2_decoder_buffer(self.h, 0, 1))
        vocab = self.s.shape.vocab
        return self.s.be.download(buf, 8 * self.generated * vocab, dtype=np.int64).reshape(self.generated, vocab)

    def cache(self, layer: int, kv: int, rows: int) -> np.ndarray:
        buf = int(self.L.vzh_gpt2_decoder_buffer(self.h, layer, 3 + kv))
        return self.s.be.download(buf, 2 * rows * self.s.shape.d, dtype=np.int16)

    def error_word(self) -> int:
        buf = int(self.L.vzh_gpt2_decoder_buffer(self.h, 0, 2))
        return int(self.s.be.download(buf, 4, dtype=np.uint32)[0])


class Gpt2Prover:
    """The prefill proof schedule over a Gpt2Session's witness, and the band
    proofs of decode chunks over the same session (libvolta_accel.so
    vzh_gpt2_prove / vzh_gpt2_prove_band; volta_zk_b200/host/gpt2_proof.cpp)."""

    def __init__(self, session: Gpt2Session):
        from . import accel

        self.s, self.host = session, session.host
        L = self.host
        L.vzh_gpt2_prover_open.restype = C.c_void_p
        L.vzh_gpt2_prover_open.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
        L.vzh_gpt2_prover_close.argtypes = [C.c_void_p]
        L.vzh_gpt2_prove.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_char_p, C.c_void_p, C.c_size_t,
                                     C.POINTER(C.c_size_t), C.POINTER(C.c_size_t), C.c_void_p, C.c_char_p,
                                     C.c_size_t]
        L.vzh_gpt2_prove_layers.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_char_p, C.c_size_t, C.c_size_t,
                                            C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t),
                                            C.POINTER(C.c_size_t), C.c_void_p, C.c_char_p, C.c_size_t]
        L.vzh_gpt2_prove_band.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_char_p, C.c_char_p, C.c_size_t,
                                          C.c_size_t, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t),
                                          C.POINTER(C.c_size_t), C.c_char_p, C.c_size_t]
        L.vzh_gpt2_prove_units.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_char_p, C.c_void_p, C.c_void_p,
                                           C.c_size_t, C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t),
                                           C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t), C.c_void_p,
                                           C.c_void_p, C.c_char_p, C.c_size_t]
        L.vzh_gpt2_correction.restype = C.c_uint64
        L.vzh_gpt2_correction.argtypes = [C.c_void_p, C.c_size_t, C.c_int]
        self._rows = session.t  # rows of the last proof (the corrections' height)
        err = C.create_string_buffer(1024)
        self.h = L.vzh_gpt2_prover_open(session.h, err, 1024)
        if not self.h:
            raise accel.AccelError(err.value.decode())
        self.cap = 1 << 20  # words (12 layers at T = 1024 take about 121 k)
        self._out = np.zeros((self.cap, 2), dtype=np.uint64)

    def close(self):
        if self.h:
            self.host.vzh_gpt2_prover_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def prove(self, seed: bytes, mac_seed: bytes, pad_seed: bytes, first: int = 0, stride: int = 1,
              with_pcs: bool = True):
        """Returns (words as an (n, 2) u64 array, words per layer, 32-byte PCS
        root).  first/stride: prove layers first, first + stride, ... only
        (one GPU's share of a proof split by layers); with_pcs: also the
        weight commitment (root all zero otherwise)."""
        from . import accel

        out = self._out
        written, per_layer = C.c_size_t(0), C.c_size_t(0)
        root = (C.c_uint8 * 32)()
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_gpt2_prove_layers(self.h, seed, mac_seed, pad_seed, first, stride, int(with_pcs),
                                             out.ctypes.data, self.cap, C.byref(written), C.byref(per_layer), root,
                                             err, 1024)
        if rc != 0:
            raise accel.AccelError(err.value.decode())
        self._rows = self.s.t
        return out[:written.value].copy(), per_layer.value, bytes(root)

    def prove_units(self, seed: bytes, mac_seed: bytes, pad_seed: bytes, units, with_pcs: bool = False):
        """Prove the units [(layer, site mask)] only, in that order (one GPU's
        share of a proof split by sites; bit k of a mask is site k, bit 0 the
        layer's boundary corrections, SITE_ORDER the rest).  Returns (words as
        an (n, 2) u64 array, per unit the list of (site, word count) in word
        order, 32-byte PCS root or zeros)."""
        from . import accel

        units = list(units)
        layers = np.array([u[0] for u in units], dtype=np.uint64)
        masks = np.array([u[1] for u in units], dtype=np.uint32)
        site_cap = 32 * max(1, len(units))
        sid, swords = np.zeros(site_cap, np.uint32), np.zeros(site_cap, np.uint64)
        per_unit = np.zeros(max(1, len(units)), np.uint64)
        out = self._out
        written, n_sites = C.c_size_t(0), C.c_size_t(0)
        root = (C.c_uint8 * 32)()
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_gpt2_prove_units(self.h, seed, mac_seed, pad_seed, layers.ctypes.data, masks.ctypes.data,
                                            len(units), int(with_pcs), out.ctypes.data, self.cap, C.byref(written),
                                            sid.ctypes.data, swords.ctypes.data, site_cap, C.byref(n_sites),
                                            per_unit.ctypes.data, root, err, 1024)
        if rc != 0:
            raise accel.AccelError(err.value.decode())
        self._rows = self.s.t
        sites, k = [], 0
        for u in range(len(units)):
            n = int(per_unit[u])
            sites.append([(int(sid[k + i]), int(swords[k + i])) for i in range(n)])
            k += n
        return out[:written.value].copy(), sites, bytes(root)

    def prove_band(self, band: "Gpt2Band", chunk: int, seed: bytes, mac_seed: bytes, first: int = 0,
                   stride: int = 1):
        """Proof of a decode band (rows t0 .. t-1 of the session's forward;
        block_proof.rs prove_layer_phase1_band, model_proof.rs prove_response
        chunks): the layer schedule over the band's q rows with attention over
        all t0 + q keys, transcripts and mask domains of chunk (>= 1).
        Returns (words as an (n, 2) u64 array, words per layer)."""
        from . import accel

        if band.s is not self.s:
            raise accel.AccelError("the band is not of this prover's session")
        out = self._out
        written, per_layer = C.c_size_t(0), C.c_size_t(0)
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_gpt2_prove_band(self.h, band.h, chunk, seed, mac_seed, first, stride, out.ctypes.data,
                                           self.cap, C.byref(written), C.byref(per_layer), err, 1024)
        if rc != 0:
            raise accel.AccelError(err.value.decode())
        self._rows = band.q
        return out[:written.value].copy(), per_layer.value

    def commit_rows(self, pad_seed: bytes, row0: int, rows: int) -> np.ndarray:
        """One GPU's row block of the weight commitment (rows = 128 * 2^k at
        a multiple of rows): each code column's BLAKE3 chaining value over
        those rows, (2^15, 32) uint8.  The blocks of all GPUs, exchanged so
        that each GPU holds a column slab (all-to-all), give the whole
        commitment's tree (sharded.ligero_shard_tree / ligero_top_tree)."""
        from . import accel

        L = self.host
        L.vzh_gpt2_commit_rows.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_char_p,
                                           C.c_size_t]
        out = np.zeros((1 << 15, 32), np.uint8)
        err = C.create_string_buffer(1024)
        if L.vzh_gpt2_commit_rows(self.h, pad_seed, row0, rows, out.ctypes.data, err, 1024) != 0:
            raise accel.AccelError(err.value.decode())
        return out

    def set_correction_sink(self, host) -> None:
        """Every later proof copies its boundary corrections into `host`
        (a contiguous u64 array of layers x 5 x rows x d, pinned for the
        copies to overlap the proof; wire w of layer l at [l, w]) while its
        later layers compute; they have landed when prove returns.  None
        stops the copies.  The array must outlive the proofs that fill it."""
        self.host.vzh_gpt2_set_correction_sink.argtypes = [C.c_void_p, C.c_void_p]
        self._sink = host
        self.host.vzh_gpt2_set_correction_sink(self.h, None if host is None else host.ctypes.data)

    def pcs_rows(self) -> int:
        """Rows of the weight commitment: 8192 while the weights fit, else
        the power of two they fill."""
        self.host.vzh_gpt2_prover_pcs_rows.restype = C.c_size_t
        self.host.vzh_gpt2_prover_pcs_rows.argtypes = [C.c_void_p]
        return int(self.host.vzh_gpt2_prover_pcs_rows(self.h))

    def host_timing(self):
        """(enqueue ms, total ms): host wall time of the last proof spent
        enqueueing its launches, and in all (the device finishes within the
        total: the downloads wait for it)."""
        e, t = C.c_double(0), C.c_double(0)
        self.host.vzh_gpt2_prover_timing.argtypes = [C.c_void_p, C.POINTER(C.c_double), C.POINTER(C.c_double)]
        self.host.vzh_gpt2_prover_timing(self.h, C.byref(e), C.byref(t))
        return e.value, t.value

    def correction(self, layer: int, wire: int) -> np.ndarray:
        """Boundary corrections x - mask of wire (0 x_in, 1 k, 2 v, 3
        attn_block_out, 4 ffn_block_out) of `layer` from the last proof: rows
        x d u64 (t rows, or the band's q)."""
        buf = int(self.host.vzh_gpt2_correction(self.h, layer, wire))
        return self.s.be.download(buf, self._rows * self.s.shape.d * 8, dtype=np.uint64)

def _lpt(items, world):
    """Largest first onto the least-loaded GPU: items [(cost, key)] ->
    (per GPU the keys, makespan)."""
    load = [0.0] * world
    keys = [[] for _ in range(world)]
    for c, key in sorted(items, key=lambda x: (-x[0], x[1])):
        g = min(range(world), key=lambda r: (load[r], r))
        load[g] += c
        keys[g].append(key)
    return keys, max(load)


def split_sites(world: int, t: int = None, layers: int = LAYERS, costs=None):
    """Deterministic split of a proof over `world` GPUs: whole layers, the
    weight commitment and, where finer units shorten the slowest GPU, the
    last k layers as their two parts (PART_ATTENTION, PART_REST), dealt
    largest first onto the least-loaded GPU with the measured costs
    (LAYER_COST, PART_COSTS, COMMIT_COST, or costs = (layer, {part: cost},
    commitment) for another shape; a commitment cost of 0 leaves it out);
    the k with the shortest slowest GPU wins, fewer splits on a tie.
    Returns (per rank the units [(layer, site mask)] in layer order, the
    rank that commits)."""
    layer_cost, part_costs, commit_cost = costs or (LAYER_COST, PART_COSTS, COMMIT_COST)
    best = None
    for k in range(layers + 1):
        items = [(commit_cost, (-1, 0))] if commit_cost else []
        items += [(layer_cost, (l, ALL_SITES)) for l in range(layers - k)]
        items += [(part_costs[m], (l, m)) for l in range(layers - k, layers) for m in (PART_ATTENTION, PART_REST)]
        keys, span = _lpt(items, world)
        if best is None or span < best[0] - 1e-9:
            best = (span, keys)
    per_rank, commit = [], 0
    for g, ks in enumerate(best[1]):
        masks = {}
        for l, m in ks:
            if l < 0:
                commit = g
            else:
                masks[l] = masks.get(l, 0) | m
        per_rank.append(sorted(masks.items()))
    return per_rank, commit


def split_span(per_rank, commit, costs=None) -> float:
    """The slowest GPU's cost of a split by the cost model (a rank holding
    both parts of a layer pays the parts); commit None: no commitment unit."""
    layer_cost, part_costs, commit_cost = costs or (LAYER_COST, PART_COSTS, COMMIT_COST)
    cost = {ALL_SITES: layer_cost, **part_costs}
    return max(sum(cost[m] for _, m in units) + (commit_cost if g == commit else 0.0)
               for g, units in enumerate(per_rank))


def split_plan(world: int, layers: int = LAYERS, costs=None, exchange_ms: float = 1.0):
    """The split of a proof over `world` GPUs with the weight commitment
    either as one GPU's unit (split_sites) or, where that is not slower by
    the cost model, split by rows over every GPU (each pays 1/world of it plus
    exchange_ms for the chaining-value all-to-all and the root gather; world
    a power of two).  Returns (per rank the units, the committing rank or
    None when every rank commits its row block)."""
    costs = costs or (LAYER_COST, PART_COSTS, COMMIT_COST)
    whole, commit = split_sites(world, layers=layers, costs=costs)
    if world == 1 or world & (world - 1):
        return whole, commit
    rows_split, _ = split_sites(world, layers=layers, costs=(costs[0], costs[1], 0))
    sharded = split_span(rows_split, None, costs) + costs[2] / world + exchange_ms
    if sharded <= split_span(whole, commit, costs) + 1e-9:  # a tie goes to the row split (measured faster)
        return rows_split, None
    return whole, commit


def assemble_units(pieces, layers: int = LAYERS):
    """The proof words of every layer in site order from the units' words:
    pieces = [(units [(layer, mask)], words, per-unit [(site, count)])] from
    every GPU.  Returns the (n, 2) u64 words in layer order."""
    by_site = {}
    for units, words, sites in pieces:
        at = 0
        for (layer, _), us in zip(units, sites):
            for site, n in us:
                by_site[(layer, site)] = words[at:at + n]
                at += n
    out = [by_site[(l, k)] for l in range(layers) for k in SITE_ORDER]
    return np.concatenate(out) if out else np.zeros((0, 2), np.uint64)


def main(argv=None):
    """One GPT-2 prefill proof on the first GPU: the synthetic model, the
    witness forward of `--tokens` prefill tokens and the proof of every layer
    plus the weight commitment (`--proofs` times); prints the proof digest."""
    import argparse
    import hashlib

    from . import accel

    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--tokens", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=None, help="default: the shape's layer count")
    ap.add_argument("--proofs", type=int, default=1)
    ap.add_argument("--scaled", action="store_true", help="the 24-layer d-1024 shape instead of GPT-2 small")
    args = ap.parse_args(argv)
    model = synthetic_model(n_layers=args.layers, shape=GPT2_SCALED if args.scaled else GPT2_SMALL)
    seeds = bytes([0x50] * 32), bytes([0x4D] * 32), bytes([0x11] * 32)
    with accel.Prover(policy=1) as prover, Gpt2Session(prover, model, args.tokens) as s, Gpt2Prover(s) as gp:
        s.forward(prefill_tokens(args.tokens))
        for _ in range(args.proofs):
            s.forward()
            words, per_layer, root = gp.prove(*seeds)
    print(f"proof words {words.shape[0]} ({per_layer} per layer), sha256 "
          f"{hashlib.sha256(words.tobytes() + root).hexdigest()[:16]}")


if __name__ == "__main__":
    main()
