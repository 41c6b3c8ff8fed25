"""ctypes bindings of the C ABI and of the host mirror.

``CudaBackend`` exposes every ``volta_cuda_*`` entry point of
``libvolta_cuda_backend.so`` with argument types parsed from
``include/volta_cuda_backend.h`` (the declarations the reference's Rust FFI
binds, rust/volta-accel/src/cuda.rs:121-974), and checks return codes the way
the seam does (``AccelError`` carrying ``volta_cuda_last_error``).

``Prover`` drives the resident protocol callers implemented in
``libvolta_accel.so`` (triple-product sumcheck, LogUp prove).

Nothing here falls back to the CPU: a missing library, a missing symbol, an
ABI mismatch or a host without a CUDA device raises ``AccelError``.
"""

from __future__ import annotations

import ctypes as C
import os
import re
from typing import Dict

import numpy as np

from .build import HERE, library_path

ROOT = os.path.dirname(HERE)
HEADER = os.path.join(ROOT, "include", "volta_cuda_backend.h")
EXT_HEADER = os.path.join(ROOT, "include", "volta_b200_ext.h")
ABI_VERSION = 37
P = 0xFFFFFFFF00000001


class AccelError(RuntimeError):
    pass


class Fp2(C.Structure):
    """Fp2Repr {c0, c1} (rust/volta-accel/src/lib.rs:394-399)."""

    _fields_ = [("c0", C.c_uint64), ("c1", C.c_uint64)]

    def tuple(self):
        return (self.c0, self.c1)


def fp2(v) -> Fp2:
    return Fp2(int(v[0]), int(v[1]))


class BlindJob(C.Structure):
    """vzb_blind_job (include/volta_b200_ext.h): one LogUp layer's blind
    corrections; 112 bytes, lambda 16-byte aligned as vz_fp2 is."""

    _fields_ = [(n, C.c_uint64) for n in (
        "raw_id raw_offset root_id root_offset sched_id sched_offset mask_id mask_offset out_id "
        "out_offset").split()] + [("lambda_", Fp2), ("rounds", C.c_uint64), ("_pad", C.c_uint64)]


assert C.sizeof(BlindJob) == 112


class RawStats(C.Structure):
    _fields_ = (
        [("calls", C.c_uint64 * 7), ("kernel_ns", C.c_uint64 * 7)]
        + [(n, C.c_uint64) for n in (
            "h2d_bytes d2h_bytes d2d_bytes device_zeroed_bytes device_generated_bytes h2d_ns d2h_ns "
            "resident_h2d_host_calls resident_d2h_host_calls resident_h2d_host_call_ns "
            "resident_d2h_host_call_ns synchronizations synchronization_ns sync_host_output "
            "sync_upload_lifetime sync_timing_flush sync_profiling_legacy sync_allocator_flush "
            "allocation_calls resident_alloc_requests resident_reuse_hits resident_free_requests "
            "physical_free_calls live_device_bytes peak_device_bytes pinned_allocation_calls "
            "pinned_alloc_requests pinned_reuse_hits pinned_free_requests pinned_physical_free_calls "
            "pinned_host_write_calls pinned_host_write_bytes live_pinned_bytes peak_pinned_bytes "
            "x4c_arena_reset_calls x4c_arena_reset_bytes x4c_kernel_launches x4c_control_peek_calls "
            "x4c_control_peek_pending timing_records timing_elapsed_query_attempts "
            "timing_elapsed_no_write timing_event_queries timing_event_api_calls "
            "timing_pending_high_water timing_flush_count coarse_timing_scopes coarse_timing_ns"
        ).split()]
        + [("timing_mode", C.c_uint32), ("reserved", C.c_uint32)]
    )


assert C.sizeof(RawStats) == 504

_CTYPES = {
    "void*": C.c_void_p, "void**": C.POINTER(C.c_void_p), "const void*": C.c_void_p,
    "uint64_t": C.c_uint64, "size_t": C.c_size_t, "int": C.c_int, "uint32_t": C.c_uint32,
    "int32_t": C.c_int32, "uint8_t": C.c_uint8, "const uint8_t*": C.c_void_p, "uint8_t*": C.c_void_p,
    "const int16_t*": C.c_void_p, "int16_t*": C.c_void_p, "const uint64_t*": C.c_void_p,
    "uint64_t*": C.c_void_p, "int64_t*": C.c_void_p, "const uint32_t*": C.c_void_p,
    "const uint16_t*": C.c_void_p, "size_t*": C.c_void_p, "int*": C.c_void_p,
    "vz_fp2": Fp2, "vz_fp2*": C.c_void_p, "const vz_fp2*": C.c_void_p,
    "vz_raw_stats*": C.c_void_p, "vz_raw_pinned_stats*": C.c_void_p,
    "vz_raw_control_state*": C.c_void_p, "const vz_attention_wires_args*": C.c_void_p,
    "float*": C.POINTER(C.c_float), "const vzb_layer_job*": C.c_void_p, "const vzb_round_job*": C.c_void_p,
    "const vzb_suffix_job*": C.c_void_p, "const vzb_blind_job*": C.c_void_p, "const vzb_copy_seg*": C.c_void_p, "const vzb_upload*": C.c_void_p,
}
_RESTYPES = {"int": C.c_int, "uint32_t": C.c_uint32, "void": None, "const char*": C.c_char_p}


def parse_header(path: str = HEADER, prefix: str = "volta_cuda_") -> Dict[str, tuple]:
    """name -> (restype, [argtypes]) for every declaration in the header."""
    text = re.sub(r"/\*.*?\*/", "", open(path).read(), flags=re.S)
    out = {}
    for ret, name, args in re.findall(
            r"\b(int|uint32_t|void|const char\*) (" + prefix + r"\w+)\(([^;]*?)\);", text, re.S):
        types = []
        args = " ".join(args.split())
        if args and args != "void":
            for a in args.split(","):
                a = a.strip()
                m = re.match(r"(.*?)(\w+)$", a)
                t = m.group(1).replace(" *", "*").strip()
                types.append(_CTYPES[t])
        out[name] = (_RESTYPES[ret], types)
    return out


_cuda_lib = None
_host_lib = None


def load_cuda_library(path: str | None = None):
    """dlopen + ABI check + eager symbol resolution (cuda.rs:1119-1170)."""
    global _cuda_lib
    if _cuda_lib is not None and path is None:
        return _cuda_lib
    path = path or os.environ.get("VOLTA_CUDA_LIBRARY") or library_path()
    if not os.path.exists(path):
        raise AccelError(f"LibraryLoad: {path} not found (build with volta_zk_b200.build_all())")
    lib = C.CDLL(path, mode=os.RTLD_NOW | os.RTLD_LOCAL)
    for name, (res, args) in parse_header().items():
        try:
            fn = getattr(lib, name)
        except AttributeError as e:
            raise AccelError(f"MissingSymbol: {name}") from e
        fn.restype = res
        fn.argtypes = args
    # extensions (include/volta_b200_ext.h): optional, as for the host
    # library, so a backend built without the newer ones still loads
    for name, (res, args) in parse_header(EXT_HEADER, "volta_b200_").items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    if lib.volta_cuda_abi_version() != ABI_VERSION:
        raise AccelError(f"AbiMismatch: expected {ABI_VERSION}, found {lib.volta_cuda_abi_version()}")
    _cuda_lib = lib
    return lib


def load_host_library():
    global _host_lib
    if _host_lib is None:
        path = library_path("libvolta_accel.so")
        if not os.path.exists(path):
            raise AccelError(f"LibraryLoad: {path} not found (build with volta_zk_b200.build_all())")
        L = C.CDLL(path)
        vp, sz, u64 = C.c_void_p, C.c_size_t, C.c_uint64
        L.vzh_open.restype = vp
        L.vzh_open.argtypes = [C.c_char_p, C.c_int, C.c_char_p, sz]
        L.vzh_close.argtypes = [vp]
        L.vzh_set_fused.argtypes = [vp, C.c_int]
        L.vzh_set_scheduled.argtypes = [vp, C.c_int]
        L.vzh_set_batched.argtypes = [vp, C.c_int]
        L.vzh_context.restype = vp
        L.vzh_context.argtypes = [vp]
        L.vzh_stats.argtypes = [vp, vp, C.c_char_p, sz]
        L.vzh_reset_stats.argtypes = [vp, C.c_char_p, sz]
        L.vzh_triple_sumcheck.argtypes = [vp, u64, u64, u64, sz, C.c_char_p, vp, vp, C.c_char_p, sz]
        L.vzh_triple_sumcheck_fp.argtypes = [vp, u64, u64, u64, sz, C.c_char_p, vp, vp, C.c_char_p, sz]
        L.vzh_triple_sumcheck_fp_host.argtypes = [vp, u64, u64, u64, vp, vp, vp, sz, sz, C.c_char_p, vp, vp,
                                                  C.c_char_p, sz]
        L.vzh_logup_prove.argtypes = [vp, u64, sz, u64, sz, u64, C.c_char_p, u64, vp, sz,
                                      C.POINTER(C.c_size_t), C.c_char_p, sz]
        L.vzh_ligero_commit_open.argtypes = [vp, C.c_char_p, sz, sz, sz, sz, C.c_char_p, vp, vp, vp, vp,
                                             C.c_char_p, sz]
        L.vzh_proof_local.argtypes = [vp, u64, u64, u64, sz, C.c_int, C.c_char_p, u64, sz, u64, sz, u64, sz,
                                      C.c_char_p, u64, vp, sz, C.POINTER(C.c_size_t), C.c_char_p, sz]
        L.vzh_proof_local_host.argtypes = [vp, u64, u64, u64, vp, vp, vp, sz, sz, C.c_char_p, u64, sz, u64, sz,
                                           u64, sz, C.c_char_p, u64, vp, sz, C.POINTER(C.c_size_t), C.c_char_p,
                                           sz]
        L.vzh_logup_local.argtypes = [vp, u64, sz, u64, sz, u64, sz, C.c_char_p, u64, vp, sz,
                                      C.POINTER(C.c_size_t), C.c_char_p, sz]
        L.vzh_ligero_commit_open_zk.argtypes = [vp, vp, sz, sz, sz, sz, C.c_char_p, sz, vp, vp, vp, C.c_char_p,
                                                u64, u64, vp, sz, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                                C.c_char_p, sz]
        L.vzh_fpstream_fp2.argtypes = [C.c_char_p, u64, sz, vp]
        L.vzh_fpstream_u64.argtypes = [C.c_char_p, u64, sz, vp]
        L.vzh_fpstream_fp.argtypes = [C.c_char_p, u64, sz, vp]
        L.vzh_blake3.argtypes = [C.c_char_p, C.c_char_p, sz, vp]
        L.vzh_blake3.restype = None
        L.vzh_blind_logup_prove.argtypes = [vp, u64, sz, u64, sz, u64, C.c_char_p, C.c_char_p, u64, vp, sz,
                                            C.POINTER(C.c_size_t), vp, C.POINTER(C.c_uint64),
                                            C.POINTER(C.c_uint64), C.c_char_p, sz]
        L.vzh_blind_logup_check.argtypes = [C.c_char_p, sz, vp, sz, C.POINTER(C.c_size_t), C.c_char_p, sz]
        _host_lib = L
    return _host_lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def blake3(data: bytes, derive_key_context: str | None = None) -> bytes:
    """BLAKE3 of `data` through the host library (derive-key mode with a context)."""
    out = np.zeros(32, dtype=np.uint8)
    ctx = derive_key_context.encode() if derive_key_context is not None else None
    load_host_library().vzh_blake3(ctx, data, len(data), _ptr(out))
    return out.tobytes()


def blind_logup_check(data: bytes, max_layers: int = 256):
    """Strict decode + re-encode of BlindLogupProof wire bytes; returns the
    per-layer round counts (lookup side, then table side)."""
    rounds = np.zeros(max_layers, dtype=np.uint32)
    layers = C.c_size_t()
    err = C.create_string_buffer(1024)
    rc = load_host_library().vzh_blind_logup_check(data, len(data), _ptr(rounds), max_layers, C.byref(layers), err,
                                                   1024)
    if rc != 0:
        raise AccelError(err.value.decode())
    return [int(x) for x in rounds[: layers.value]]


class CudaBackend:
    """One resident context of libvolta_cuda_backend.so (policy 0 deferred
    events, 1 wall-only counters; None keeps the synchronous event mode)."""

    def __init__(self, policy: int | None = 0, ctx=None, lib=None):
        self.lib = lib or load_cuda_library()
        self._owned = ctx is None
        if ctx is None:
            raw = C.c_void_p()
            rc = self.lib.volta_cuda_create(C.byref(raw))
            if rc != 0:
                msg = self.lib.volta_cuda_last_error(raw).decode() if raw.value else "create failed"
                if raw.value:
                    self.lib.volta_cuda_destroy(raw)
                raise AccelError(f"Cuda: {msg}")
            self.ctx = raw
            if policy is not None:
                self.check(self.lib.volta_cuda_set_resident_timing_policy(self.ctx, policy),
                           "set_resident_timing_policy")
        else:
            self.ctx = C.c_void_p(ctx)

    def close(self):
        if self._owned and self.ctx:
            self.lib.volta_cuda_destroy(self.ctx)
            self.ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def last_error(self) -> str:
        return self.lib.volta_cuda_last_error(self.ctx).decode()

    def check(self, rc: int, what: str):
        if rc != 0:
            raise AccelError(f"Cuda: {what}: {self.last_error()} (rc={rc})")

    def call(self, name: str, *args):
        fn = getattr(self.lib, "volta_cuda_" + name)
        self.check(fn(self.ctx, *args), name)

    # ---- arena -----------------------------------------------------------------
    def alloc(self, nbytes: int) -> int:
        out = C.c_uint64()
        self.check(self.lib.volta_cuda_resident_alloc(self.ctx, max(int(nbytes), 16), C.byref(out)),
                   "resident_alloc")
        return out.value

    def free(self, buf: int):
        self.check(self.lib.volta_cuda_resident_free(self.ctx, buf), "resident_free")

    def upload(self, buf: int, array: np.ndarray, offset_bytes: int = 0):
        a = np.ascontiguousarray(array)
        self.check(self.lib.volta_cuda_resident_upload(self.ctx, buf, offset_bytes, _ptr(a), a.nbytes),
                   "resident_upload")

    def download(self, buf: int, nbytes: int, dtype=np.uint64, offset_bytes: int = 0) -> np.ndarray:
        out = np.zeros(nbytes // np.dtype(dtype).itemsize, dtype=dtype)
        self.check(self.lib.volta_cuda_resident_download(self.ctx, buf, offset_bytes, _ptr(out), nbytes),
                   "resident_download")
        return out

    def upload_new(self, array: np.ndarray) -> int:
        a = np.ascontiguousarray(array)
        buf = self.alloc(a.nbytes)
        self.upload(buf, a)
        return buf

    def download_fp2(self, buf: int, n: int, offset: int = 0) -> np.ndarray:
        return self.download(buf, 16 * n, offset_bytes=16 * offset).reshape(n, 2)

    def stats(self) -> RawStats:
        s = RawStats()
        self.check(self.lib.volta_cuda_get_stats(self.ctx, C.byref(s)), "get_stats")
        return s

    # ---- asynchronous uploads (extension) --------------------------------------
    def upload_async(self, buf: int, src_ptr: int, nbytes: int, offset_bytes: int = 0):
        """Copy nbytes from host address src_ptr (pinned for a truly
        asynchronous copy) on the context's copy stream; see wait_uploads."""
        self.check(self.lib.volta_b200_upload_async(self.ctx, buf, offset_bytes, C.c_void_p(src_ptr), nbytes),
                   "upload_async")

    def wait_uploads(self):
        """Later work on this context waits for every upload_async so far."""
        self.check(self.lib.volta_b200_wait_uploads(self.ctx), "wait_uploads")

    def embed_i16(self, in_buf: int, out_buf: int, n: int):
        """out[i] = int16 in[i] embedded in Fp (canonical), on the device."""
        self.check(self.lib.volta_b200_embed_i16_device(self.ctx, in_buf, 0, out_buf, 0, n), "embed_i16")

    # ---- measurement extensions ---------------------------------------------
    def mark(self, slot: int):
        self.check(self.lib.volta_b200_timing_mark(self.ctx, slot), "timing_mark")

    def elapsed_ms(self, start: int, end: int) -> float:
        ms = C.c_float()
        self.check(self.lib.volta_b200_timing_elapsed(self.ctx, start, end, C.byref(ms)), "timing_elapsed")
        return ms.value

    def launches(self) -> int:
        n = C.c_uint64()
        self.check(self.lib.volta_b200_launch_count(self.ctx, C.byref(n)), "launch_count")
        return n.value


def fpstream_fp2(seed: bytes, domain: int, n: int) -> np.ndarray:
    """The first n Fp2 draws of FpStream(seed, domain), shape (n, 2)."""
    out = np.zeros((n, 2), dtype=np.uint64)
    load_host_library().vzh_fpstream_fp2(seed, domain, n, _ptr(out))
    return out


def fpstream_fp_rows(seed: bytes, domain: int, n: int) -> np.ndarray:
    """The first n Fp draws of FpStream(seed, domain) (next_fp, rejection
    exact): the values chacha8_prover_secret_fp_rows_device writes for row
    `domain`."""
    out = np.zeros(n, dtype=np.uint64)
    load_host_library().vzh_fpstream_fp(seed, domain & (2**64 - 1), n, _ptr(out))
    return out


def fpstream_u64(seed: bytes, domain: int, n: int) -> np.ndarray:
    """Raw u64 draws of FpStream(seed, domain) (rust/volta-field/src/lib.rs:231-267)."""
    out = np.zeros(n, dtype=np.uint64)
    load_host_library().vzh_fpstream_u64(seed, domain & (2**64 - 1), n, _ptr(out))
    return out


class Prover:
    """Resident protocol drivers of libvolta_accel.so on their own context."""

    def __init__(self, policy: int = 1, fused: bool = True, scheduled: bool = True, batched: bool = True):
        self.host = load_host_library()
        load_cuda_library()  # same dlopen handle as the host library's
        err = C.create_string_buffer(1024)
        self.h = self.host.vzh_open(library_path().encode(), policy, err, 1024)
        if not self.h:
            raise AccelError(err.value.decode())
        self.backend = CudaBackend(ctx=self.host.vzh_context(self.h))
        self.host.vzh_set_fused(self.h, 1 if fused else 0)
        self.host.vzh_set_scheduled(self.h, 1 if scheduled else 0)
        self.host.vzh_set_batched(self.h, 1 if batched else 0)

    def close(self):
        if self.h:
            self.host.vzh_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _err(self, rc, err):
        if rc != 0:
            raise AccelError(err.value.decode())

    def triple_sumcheck(self, a: int, b: int, c: int, n: int, seed: bytes):
        rounds = n.bit_length() - 1
        msgs = np.zeros((3 * rounds, 2), dtype=np.uint64)
        finals = np.zeros((3, 2), dtype=np.uint64)
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_triple_sumcheck(self.h, a, b, c, n, seed, _ptr(msgs), _ptr(finals), err, 1024)
        self._err(rc, err)
        return msgs, finals

    def triple_sumcheck_fp(self, a: int, b: int, c: int, n: int, seed: bytes):
        """The same proof on three resident columns of n canonical Fp values
        (tables whose c1 is 0), without lifting them to Fp2 first."""
        rounds = n.bit_length() - 1
        msgs = np.zeros((3 * rounds, 2), dtype=np.uint64)
        finals = np.zeros((3, 2), dtype=np.uint64)
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_triple_sumcheck_fp(self.h, a, b, c, n, seed, _ptr(msgs), _ptr(finals), err, 1024)
        self._err(rc, err)
        return msgs, finals

    def triple_sumcheck_fp_host(self, a: int, b: int, c: int, host, n: int, seed: bytes, chunk: int = 0):
        """triple_sumcheck_fp with the columns still in host memory: `host`
        holds three host addresses (pinned, n u64 each) whose values fill the
        device columns a, b, c chunk by chunk (chunk entries per column, 0 for
        the default) while the first rounds prove the chunks that have landed."""
        rounds = n.bit_length() - 1
        msgs = np.zeros((3 * rounds, 2), dtype=np.uint64)
        finals = np.zeros((3, 2), dtype=np.uint64)
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_triple_sumcheck_fp_host(self.h, a, b, c, host[0], host[1], host[2], n, chunk, seed,
                                                   _ptr(msgs), _ptr(finals), err, 1024)
        self._err(rc, err)
        return msgs, finals

    def logup_prove(self, f_col: int, n_f: int, t_col: int, n_t: int, mult: int, seed: bytes,
                    domain: int, cap: int):
        out = np.zeros((cap, 2), dtype=np.uint64)
        written = C.c_size_t()
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_logup_prove(self.h, f_col, n_f, t_col, n_t, mult, seed, domain, _ptr(out), cap,
                                       C.byref(written), err, 1024)
        self._err(rc, err)
        return out[: written.value]

    def blind_logup_prove(self, f_col: int, n_f: int, t_col: int, n_t: int, mult: int, tx_seed: bytes,
                          corr_seed: bytes, dom_base: int):
        """Blind LogUp proof (rust/volta-proto/src/logup.rs:3184-3225) with a
        fresh private transcript and the mock correlation stream: (proof wire
        bytes, transcript binding digest, transcript bytes, next domain)."""
        d_f, d_t = n_f.bit_length() - 1, n_t.bit_length() - 1
        cap = 4096 + 16 * 2 * (d_f * d_f + d_t * d_t + 8 * (d_f + d_t))
        out = np.zeros(cap, dtype=np.uint8)
        digest = np.zeros(32, dtype=np.uint8)
        written, tx_bytes, next_dom = C.c_size_t(), C.c_uint64(), C.c_uint64()
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_blind_logup_prove(self.h, f_col, n_f, t_col, n_t, mult, tx_seed, corr_seed, dom_base,
                                             _ptr(out), cap, C.byref(written), _ptr(digest), C.byref(tx_bytes),
                                             C.byref(next_dom), err, 1024)
        self._err(rc, err)
        return out[: written.value].tobytes(), digest.tobytes(), tx_bytes.value, next_dom.value

    def ligero_commit_open(self, row_seed: bytes, rows: int, msg_len: int, code_len: int, queries: int,
                           chal_seed: bytes):
        """Commit seeded message rows and open `queries` columns: (root bytes,
        indices, columns [queries x rows], paths [queries x log2(code_len) x 32])."""
        bits = code_len.bit_length() - 1
        root = np.zeros(32, dtype=np.uint8)
        idx = np.zeros(queries, dtype=np.uint32)
        cols = np.zeros((queries, rows), dtype=np.uint64)
        paths = np.zeros((queries, bits, 32), dtype=np.uint8)
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_ligero_commit_open(self.h, row_seed, rows, msg_len, code_len, queries, chal_seed,
                                              _ptr(root), _ptr(idx), _ptr(cols), _ptr(paths), err, 1024)
        self._err(rc, err)
        return root.tobytes(), idx, cols, paths

    def logup_local(self, f_col: int, n_f_local: int, t_col: int, n_t_local: int, mult: int, shard_bits: int,
                    seed: bytes, domain: int) -> np.ndarray:
        """This shard's share of a LogUp proof (see vzh_logup_local): Fp2 words."""
        cap = 1 + 2 * (2 + sum(4 * (l - shard_bits) + 4 for l in range(shard_bits, 64)))
        out = np.zeros((cap, 2), dtype=np.uint64)
        written = C.c_size_t()
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_logup_local(self.h, f_col, n_f_local, t_col, n_t_local, mult, shard_bits, seed, domain,
                                       _ptr(out), cap, C.byref(written), err, 1024)
        self._err(rc, err)
        return out[: written.value]

    def proof_local(self, a: int, b: int, c: int, n_local: int, base: bool, triple_seed: bytes, f_col: int,
                    n_f_local: int, t_col: int, n_t_local: int, mult: int, shard_bits: int, logup_seed: bytes,
                    domain: int, host=None, chunk: int = 0) -> np.ndarray:
        """This shard's whole config-1 part in one call (vzh_proof_local): the
        triple sumcheck words (3 k messages, 3 finals) then the LogUp local
        words, with a single download for both.  With `host` (three host
        addresses of pinned Fp columns, base only), the triple columns a, b, c
        are filled from host memory chunk by chunk while the LogUp part and the
        first triple rounds compute (vzh_proof_local_host)."""
        k = n_local.bit_length() - 1
        cap = 3 * k + 3 + 1 + 2 * (2 + sum(4 * (l - shard_bits) + 4 for l in range(shard_bits, 64)))
        out = np.zeros((cap, 2), dtype=np.uint64)
        written = C.c_size_t()
        err = C.create_string_buffer(1024)
        if host is not None:
            if not base:
                raise AccelError("host columns need base-field tables")
            rc = self.host.vzh_proof_local_host(self.h, a, b, c, host[0], host[1], host[2], chunk, n_local,
                                                triple_seed, f_col, n_f_local, t_col, n_t_local, mult, shard_bits,
                                                logup_seed, domain, _ptr(out), cap, C.byref(written), err, 1024)
        else:
            rc = self.host.vzh_proof_local(self.h, a, b, c, n_local, 1 if base else 0, triple_seed, f_col,
                                           n_f_local, t_col, n_t_local, mult, shard_bits, logup_seed, domain,
                                           _ptr(out), cap, C.byref(written), err, 1024)
        self._err(rc, err)
        return out[: written.value]

    def ligero_commit_open_zk(self, weights: np.ndarray, rows: int, col_bits: int, pad: int, code_bits: int,
                              pad_seed: bytes, claims, mask_seed: bytes, c, indices):
        """Weight-matrix commitment and the device part of its zero-knowledge
        multi-claim opening (vzh_ligero_commit_open_zk; ligero.rs:465-505,
        1187-1480).  weights: rows x 2^col_bits int16; claims: [(offset,
        point [k x 2] u64)]; c: the proximity challenge (c0, c1); indices: the
        query columns.  Returns a dict of root, mask_root, u_c, u_g, s,
        columns, mask_columns, paths, mask_paths and the host-timed phases."""
        w = np.ascontiguousarray(weights, dtype=np.int16)
        n, q = len(claims), len(indices)
        cols, msg_len = 1 << col_bits, (1 << col_bits) + pad
        offsets = np.array([cl[0] for cl in claims], dtype=np.uint64)
        lens = np.array([len(cl[1]) for cl in claims], dtype=np.uint64)
        pts = np.ascontiguousarray(np.concatenate([np.asarray(cl[1], dtype=np.uint64).reshape(-1, 2)
                                                   for cl in claims]) if claims else np.zeros((0, 2)),
                                   dtype=np.uint64)
        idx = np.ascontiguousarray(indices, dtype=np.uint32)
        out = {"root": np.zeros(32, np.uint8), "mask_root": np.zeros(32, np.uint8),
               "u_c": np.zeros((msg_len, 2), np.uint64), "u_g": np.zeros((n * msg_len, 2), np.uint64),
               "s": np.zeros((n, 2), np.uint64), "columns": np.zeros(q * rows, np.uint64),
               "mask_columns": np.zeros((q * (n + 1), 2), np.uint64),
               "paths": np.zeros(q * code_bits * 32, np.uint8), "mask_paths": np.zeros(q * code_bits * 32, np.uint8)}
        phases = np.zeros(2, np.float64)
        err = C.create_string_buffer(1024)
        rc = self.host.vzh_ligero_commit_open_zk(
            self.h, _ptr(w), rows, col_bits, pad, code_bits, pad_seed, n, _ptr(offsets), _ptr(lens), _ptr(pts),
            mask_seed, int(c[0]), int(c[1]), _ptr(idx), q, _ptr(out["root"]), _ptr(out["mask_root"]),
            _ptr(out["u_c"]), _ptr(out["u_g"]), _ptr(out["s"]), _ptr(out["columns"]), _ptr(out["mask_columns"]),
            _ptr(out["paths"]), _ptr(out["mask_paths"]), _ptr(phases), err, 1024)
        self._err(rc, err)
        out["commit_ms"], out["open_ms"] = float(phases[0]), float(phases[1])
        return out

    def stats(self) -> RawStats:
        return self.backend.stats()
