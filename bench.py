#!/usr/bin/env python3
"""Benchmark: VOLTA-ZK's prover hot path on B200 through the drop-in C ABI.

Headline (BASELINE metric, config 3): the GPT-2 small prefill proof of
T = 1024 tokens.  One step = the int16 witness forward (embed, 12 layers,
final LN, logits of the last position) + the prefill proof schedule over
that witness (per layer: 14 LogUp lookup instances, the weight-GEMM,
attention and LayerNorm/softmax product sumchecks, VOLE-MAC boundary
corrections) + the Ligero commitment of the weights.  Model: the reference's
synthetic_model (rust/volta-gpt2/src/model.rs:504-600, seed 0x1234), token
ids FpStream([0x70;32], 0).next_fp() mod 50257.  value = seconds per proof;
rho = proof / the plain int16 forward (docs/benchmark-plan.md:10-20).

Also in the line: config 1 (triple-product sumcheck over three 2^24 tables
+ LogUp of 2^24 GELU-table queries), config 2 (Ligero commitment 8192 x
2^14 -> 2^16, 128 openings), the GPT2_FULL zero-knowledge commitment and the
witness GEMMs.  Inputs are synthetic (no dataset exists for these
workloads).

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                       [--workload config3|config1]
Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GPT-2s 1024-tok prefill prove s & rho at 1/2/4/8 B200; kernel GB/s vs HBM peak"
P = 0xFFFFFFFF00000001
SUMCHECK_SEED = bytes([0x51] * 32)
TRANSCRIPT_SEED = bytes([0x5A] * 32)
LOGUP_SEED = bytes([0x4C] * 32)
LOGUP_DOMAIN = 0x1004
LIGERO_ROW_SEED = bytes([0x11] * 32)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["config3", "config1"], default="config3",
                    help="config3: GPT-2 small prefill proof (the metric); config1: the standalone sumcheck + LogUp")
    ap.add_argument("--tokens", type=int, default=1024, help="config 3 prefill length")
    ap.add_argument("--no-config1", action="store_true", help="config 3 line without the config-1 sub-object")
    ap.add_argument("--log2-sumcheck", type=int, default=24)
    ap.add_argument("--log2-queries", type=int, default=24)
    ap.add_argument("--log2-table", type=int, default=16)
    ap.add_argument("--ligero-rows", type=int, default=8192)
    ap.add_argument("--ligero-log2-msg", type=int, default=14)
    ap.add_argument("--ligero-log2-code", type=int, default=16)
    ap.add_argument("--ligero-queries", type=int, default=128)
    ap.add_argument("--no-ligero", action="store_true")
    ap.add_argument("--no-ligero-zk", action="store_true")
    ap.add_argument("--split-gather", action="store_true",
                    help="N > 1, two lanes: the LogUp lane gathers on a second NCCL communicator as soon as its "
                         "local part is done")
    ap.add_argument("--no-gemm", action="store_true")
    ap.add_argument("--lanes", type=int, choices=[1, 2], default=2,
                    help="2: the triple sumcheck and the LogUp proof run concurrently on two contexts")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="config 3 line without the config-4 witness leg")
    ap.add_argument("--no-scaled", action="store_true", help="config 3 line without the config-4 scaled-shape leg")
    ap.add_argument("--commit", choices=["auto", "unit", "rows"], default="auto",
                    help="weight commitment at N > 1: by the cost model, on one GPU, or split by rows")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# workload synthesis (shared by both arms; host side, untimed)
# ---------------------------------------------------------------------------

def gelu_table() -> np.ndarray:
    """The 2^16-entry int16 GELU table of luts.rs build_luts (LutParams
    defaults), indexed by the input's u16 bit pattern."""
    from volta_zk_b200.gpt2 import build_luts

    return build_luts()["gelu"]


def embed_i16(v: np.ndarray) -> np.ndarray:
    v64 = v.astype(np.int64)
    return np.where(v64 >= 0, v64.astype(np.uint64), np.uint64(P) - (-v64).astype(np.uint64)).astype(np.uint64)


def logup_inputs(log2_queries: int, log2_table: int, draw_u64):
    table = gelu_table()[: 1 << log2_table] if log2_table < 16 else gelu_table()
    raw = draw_u64(LOGUP_SEED, 1, 1 << log2_queries)
    idx = (raw & np.uint64((1 << log2_table) - 1)).astype(np.int64)
    f = table[idx]
    mult = np.bincount(idx, minlength=1 << log2_table).astype(np.uint32)
    return f, table, mult


def proof_words(n_f: int, n_t: int) -> int:
    def side(n):
        d = n.bit_length() - 1
        return 2 + sum(2 * l + 4 for l in range(d))

    return 1 + side(n_f) + side(n_t)


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for k, n in enumerate(names):
                if len(s) > 5 + k and s[5 + k].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU baseline (the reference's CPU algorithm, C/OpenMP restatement)
# ---------------------------------------------------------------------------

def cpu_inputs(log2_sumcheck: int, log2_queries: int, log2_table: int):
    """Config-1 inputs for the CPU arm, at full size: the three FpStream
    tables lifted to Fp2 and the LogUp query/table/multiplicity columns."""
    from volta_zk_b200.accel import fpstream_fp_rows  # host ChaCha8 (input synthesis only)

    n = 1 << log2_sumcheck
    tabs = []
    for k in range(3):
        t = np.zeros((n, 2), dtype=np.uint64)
        t[:, 0] = fpstream_fp_rows(SUMCHECK_SEED, k, n)
        tabs.append(t)
    from volta_zk_b200.accel import fpstream_u64

    return tabs, logup_inputs(log2_queries, log2_table, fpstream_u64)


def cpu_prove_times(tabs, logup, steps: int):
    """The reference's CPU algorithm for one whole config-1 proof (the C/OpenMP
    oracle restatement: clear triple-product sumcheck + logup_prove) on every
    host core this process may use, timed per proof.  The thread count is set
    explicitly (torchrun exports OMP_NUM_THREADS=1 when it starts several
    processes).  Returns (seconds per proof, threads used, the last proof as
    (messages, finals, LogUp words))."""
    from oracle import oracle as o  # checker / baseline only

    o.build()
    threads = o.set_threads(o.host_threads())
    f, table, mult = logup
    times, out = [], None
    for _ in range(steps):
        t0 = time.perf_counter()
        msgs, finals = o.triple_sumcheck(*tabs, TRANSCRIPT_SEED)
        words = o.logup_prove(f, table, mult, LOGUP_SEED, LOGUP_DOMAIN)
        times.append(time.perf_counter() - t0)
        out = (msgs, finals, words)
    return times, threads, out


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------

LIGERO_MASK_SEED = bytes([0xA5] * 32)


def ligero_zk_inputs():
    """Seeded GPT2_FULL-shaped inputs of the ZK commitment leg: 8192 x 2^14
    int16 weights, 512 pads, code 2^15, 13 claims on aligned row blocks,
    challenge c and 200 query indices."""
    rows, col_bits, pad, code_bits, queries, n_claims = 8192, 14, 512, 15, 200, 13
    rng = np.random.default_rng(0x11)
    w = rng.integers(-32768, 32768, size=(rows, 1 << col_bits), dtype=np.int64).astype(np.int16)
    claims = []
    for g in range(n_claims):  # blocks of 2^k rows, aligned
        k = g % 8
        row0 = (g * 613 // (1 << k)) * (1 << k) % rows
        claims.append((row0 << col_bits, rng.integers(0, P, size=(col_bits + k, 2), dtype=np.uint64)))
    c = tuple(int(x) for x in rng.integers(0, P, size=2, dtype=np.uint64))
    idx = rng.integers(0, 1 << code_bits, size=queries).astype(np.uint32)
    return {"rows": rows, "col_bits": col_bits, "pad": pad, "code_bits": code_bits, "w": w, "claims": claims,
            "c": c, "idx": idx}


def ligero_zk_leg(prover, reps=3):
    """The reference's full-scale weight commitment shape (ligero.rs:59-60,
    GPT2_FULL: 8192 rows of 2^14 int16 weights + 512 ChaCha8 pads, RS-encoded
    to 2^15, 200 queries) committed from host weights, then the device part of
    its zero-knowledge opening for 13 claims (ligero.rs:1187-1480): 14 Fp2
    mask rows encoded and committed, the proximity row and 13 claim rows over
    the whole matrix, 13 masked row dots, 200 data and mask columns with their
    paths.  Seeded synthetic weights and claims; phases timed on the host
    around their synchronising downloads (median of `reps`)."""
    import torch

    z = ligero_zk_inputs()
    rows, col_bits, pad, code_bits = z["rows"], z["col_bits"], z["pad"], z["code_bits"]
    # the weights live in pinned host memory, as a serving process keeps them
    w = torch.from_numpy(z["w"]).pin_memory().numpy()
    runs = []
    for _ in range(reps + 1):
        o = prover.ligero_commit_open_zk(w, rows, col_bits, pad, code_bits, LIGERO_ROW_SEED, z["claims"],
                                         LIGERO_MASK_SEED, z["c"], z["idx"])
        runs.append((o["commit_ms"], o["open_ms"]))
    runs = runs[1:]
    commit_ms = float(np.median([r[0] for r in runs]))
    open_ms = float(np.median([r[1] for r in runs]))
    return {"workload": "GPT2_FULL Ligero weight commitment (8192 x 2^14 int16 + 512 pads -> 2^15) from pinned "
                        "host weights + device part of the ZK opening (13 claims, 14 mask rows, 200 queries)",
            "commit_ms": round(commit_ms, 3), "open_ms": round(open_ms, 3), "unit": "ms", "timing": "host, median",
            "root": bytes(o["root"]).hex(), "mask_root": bytes(o["mask_root"]).hex()}


def ligero_leg(args, prover, be, peaks, rank=0, world=1, comm=None):
    """Ligero commitment of rows x 2^msg seeded Fp message
    rows, RS-encoded to 2^code columns (rate 1/4 at the defaults), BLAKE3
    column Merkle tree and 128 column openings, through the host API (one
    call per commitment; the message rows are generated on the device by the
    ChaCha8 row kernel, the root, columns and paths come back to the host)."""
    rows, msg, code, q = args.ligero_rows, 1 << args.ligero_log2_msg, 1 << args.ligero_log2_code, args.ligero_queries

    def step():
        if world == 1:
            return prover.ligero_commit_open(LIGERO_ROW_SEED, rows, msg, code, q, TRANSCRIPT_SEED)
        # rows split across the GPUs, column chaining values exchanged all-to-all
        from volta_zk_b200.sharded import ligero_commit_open_sharded

        return ligero_commit_open_sharded(be, rank, world, comm[0], comm[1], LIGERO_ROW_SEED, rows, msg, code, q,
                                          TRANSCRIPT_SEED)

    for _ in range(max(1, args.warmup)):
        out = step()
    be.mark(6)
    for _ in range(args.steps):
        out = step()
    be.mark(7)
    commit_s = be.elapsed_ms(6, 7) / 1e3 / args.steps
    if world > 1:  # one commitment over all GPUs: report it without the single-GPU kernel loops
        return {"workload": f"config 2: Ligero commit {rows} rows x 2^{args.ligero_log2_msg} msg -> "
                            f"2^{args.ligero_log2_code} code, BLAKE3 column Merkle, {q} openings, rows split over "
                            f"{world} GPUs (all-to-all of 32-byte column chaining values)",
                "value": round(commit_s, 6), "unit": "s/commitment", "higher_is_better": False,
                "root": out[0].hex()}
    e2e = None if args.no_e2e else ligero_e2e(args, be, out[0])
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle as o  # checker / baseline only

        o.build()
        threads = o.set_threads(o.host_threads())
        t0 = time.perf_counter()
        ref = o.ligero_commit_open(LIGERO_ROW_SEED, rows, msg, code, q, TRANSCRIPT_SEED)
        cpu_s = time.perf_counter() - t0
        cpu = {"value": round(cpu_s, 3), "unit": "s/commitment", "cores": threads, "kind": "port",
               "sample": f"one whole config-2 commitment with its {q} openings at full size (oracle: C/OpenMP "
                         f"restatement of ligero.rs commit + open)",
               "parity": bool(ref[0] == out[0] and np.array_equal(ref[1], out[1]) and np.array_equal(ref[2], out[2])
                              and np.array_equal(ref[3], out[3]))}
    # dominant kernels alone on a resident codeword (in place, inputs >> L2)
    buf = be.alloc(8 * rows * code)
    be.call("chacha8_prover_secret_fp_rows_device", buf, 0, LIGERO_ROW_SEED, 0, rows, code)
    tree = be.alloc(32 * (2 * code - 1))
    reps = 5
    be.call("ntt_fp_batch_device", buf, 0, rows, code, buf, 0)
    be.mark(8)
    for _ in range(reps):
        be.call("ntt_fp_batch_device", buf, 0, rows, code, buf, 0)
    be.mark(9)
    be.call("hash_fp_tree_device", buf, 0, rows, code, tree, 0)
    be.mark(10)
    for _ in range(reps):
        be.call("hash_fp_tree_device", buf, 0, rows, code, tree, 0)
    be.mark(11)
    ntt_ms = be.elapsed_ms(8, 9) / reps
    hash_ms = be.elapsed_ms(10, 11) / reps
    be.free(buf)
    be.free(tree)
    data = 8 * rows * code
    hbm = peaks.get("hbm_gbs", 6650.0)
    butterflies = rows * (code // 2) * args.ligero_log2_code
    chunks = (rows * 8 + 1023) // 1024
    compressions = code * (chunks * 16 + chunks - 1) + (code - 1)
    return {
        "workload": f"config 2: Ligero commit {rows} rows x 2^{args.ligero_log2_msg} msg -> 2^{args.ligero_log2_code} "
                    f"code, BLAKE3 column Merkle, {q} openings",
        "value": round(commit_s, 6), "unit": "s/commitment", "higher_is_better": False,
        "root": out[0].hex(), "e2e": e2e, "cpu_baseline": cpu,
        "kernels": {
            "ntt_fp_batch": {"avg_launch_ms": round(ntt_ms, 4),
                             "hbm_gbs": round(2 * data / (ntt_ms / 1e3) / 1e9, 1),
                             "frac_of_hbm_peak": round(2 * data / (ntt_ms / 1e3) / 1e9 / hbm, 4),
                             "butterflies_per_s": round(butterflies / (ntt_ms / 1e3), 1),
                             "algorithmic_bytes": 2 * data,
                             "issue": issue_roofline(NTT_WARP_INST_PER_BUTTERFLY * butterflies, ntt_ms),
                             "alu_pipe_ncu": {"pass1": 0.772, "pass2": 0.849,
                                              "source": "ncu at 1024 rows x 2^16 (ALU pipe, pct of peak)"}},
            "hash_fp_tree": {"avg_launch_ms": round(hash_ms, 4),
                             "hbm_gbs": round(data / (hash_ms / 1e3) / 1e9, 1),
                             "frac_of_hbm_peak": round(data / (hash_ms / 1e3) / 1e9 / hbm, 4),
                             "blake3_compressions_per_s": round(compressions / (hash_ms / 1e3), 1),
                             "algorithmic_bytes": data,
                             "alu_pipe_ncu": {"column_leaves": 0.913,
                                              "source": "ncu at 1024 rows x 2^16 (ALU pipe, pct of peak)"}},
        },
    }


def ligero_e2e(args, be, root_resident: bytes, steps: int = 3):
    """Config 2 end to end through the seam with host buffers: the message
    rows (rows x 2^msg Fp, the same seeded rows) from pinned host memory to
    the device each step, zero-padded to the code length on the device, the
    batched NTT, the BLAKE3 column tree, the openings' columns and paths
    gathered on the device, and the root, columns and paths back to the
    host.  Returns the e2e object (its root must equal the resident run's)."""
    import torch

    from volta_zk_b200.sharded import ligero_query_indices

    rows, msg, code, q = args.ligero_rows, 1 << args.ligero_log2_msg, 1 << args.ligero_log2_code, args.ligero_queries
    bits = code.bit_length() - 1
    stage = be.alloc(8 * rows * msg)
    be.call("chacha8_prover_secret_fp_rows_device", stage, 0, LIGERO_ROW_SEED, 0, rows, msg)
    pinned = torch.empty(rows * msg, dtype=torch.int64).pin_memory()
    host = pinned.numpy().view(np.uint64)
    host[:] = be.download(stage, 8 * rows * msg)
    codeword = be.alloc(8 * rows * code)
    tree = be.alloc(32 * (2 * code - 1))
    idx = ligero_query_indices(TRANSCRIPT_SEED, q, code)
    ids = be.upload_new(idx)
    cols = be.alloc(8 * q * rows)
    paths = be.alloc(32 * q * bits)

    def step():
        be.upload(stage, host)
        be.call("resident_zero", codeword, 0, 8 * rows * code)
        be.call("resident_copy_rows", stage, 0, 8 * msg, codeword, 0, 8 * code, rows, 8 * msg)
        be.call("ntt_fp_batch_device", codeword, 0, rows, code, codeword, 0)
        be.call("hash_fp_tree_device", codeword, 0, rows, code, tree, 0)
        be.call("pcs_gather_columns_device", codeword, 0, rows, code, ids, 0, q, cols, 0, 0)
        be.call("merkle_paths_device", tree, 0, code, ids, 0, q, paths, 0)
        root = be.download(tree, 32, dtype=np.uint8, offset_bytes=32 * (2 * code - 2)).tobytes()
        return root, be.download(cols, 8 * q * rows), be.download(paths, 32 * q * bits, dtype=np.uint8)

    step()
    be.mark(12)
    for _ in range(steps):
        root, _, _ = step()
    be.mark(13)
    e2e_s = be.elapsed_ms(12, 13) / 1e3 / steps
    for b in (stage, codeword, tree, ids, cols, paths):
        be.free(b)
    return {"value": round(e2e_s, 6), "unit": "s/commitment", "h2d_bytes_per_step": 8 * rows * msg,
            "d2h_bytes_per_step": 32 + 8 * q * rows + 32 * q * bits,
            "inputs": "message rows (Fp) from pinned host memory; out: root, opened columns and their paths",
            "root_matches_resident": root == root_resident}


# GPT-2 small at 1024 tokens: QKV, attention projection, MLP up and down, logits (m, k, n)
GEMM_SHAPES = [(1024, 768, 2304), (1024, 768, 768), (1024, 768, 3072), (1024, 3072, 768), (1024, 768, 50257)]


def gemm_leg(args, be, peaks):
    """Witness GEMMs (exact int16 x int16 -> int64) of one GPT-2 small layer
    plus the logits, each through the reference's resident entry point
    volta_cuda_gemm_i64_device (byte-plane split + tcgen05 kernel).  The
    tensor-core work is 4 int8 products per int16 MAC; the peak is twice the
    measured dense bf16 rate (B200's dense int8 rate is twice its bf16
    rate)."""
    rng = np.random.default_rng(7)
    reps = max(3, args.steps)
    out, total_ms, total_ops = {}, 0.0, 0.0
    for m, k, n in GEMM_SHAPES:
        a = be.upload_new(rng.integers(-32768, 32768, m * k, dtype=np.int16))
        b = be.upload_new(rng.integers(-32768, 32768, k * n, dtype=np.int16))
        o = be.alloc(8 * m * n)
        for _ in range(max(1, args.warmup)):
            be.call("gemm_i64_device", a, 0, b, 0, o, 0, m, k, n)
        be.mark(12)
        for _ in range(reps):
            be.call("gemm_i64_device", a, 0, b, 0, o, 0, m, k, n)
        be.mark(13)
        ms = be.elapsed_ms(12, 13) / reps
        ops = 8.0 * m * k * n
        out[f"{m}x{k}x{n}"] = {"ms": round(ms, 4), "int8_tops": round(ops / (ms / 1e3) / 1e12, 1)}
        total_ms += ms
        total_ops += ops
        for x in (a, b, o):
            be.free(x)
    peak = 2 * peaks.get("bf16_tflops", 1590.0)
    achieved = total_ops / (total_ms / 1e3) / 1e12
    return {"workload": "GPT-2 small layer GEMMs + logits at 1024 tokens, exact int16 -> int64",
            "kernel": "gemm_tc_kernel (tcgen05.mma kind::i8, TMEM accumulators) + byte-plane split",
            "shapes": out, "total_ms": round(total_ms, 4),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                         "unit": "int8 TOP/s", "frac": round(achieved / peak, 4),
                         "peak_source": "2 x measured bf16 dense" if "bf16_tflops" in peaks else "2 x fallback bf16"}}


class RoundJob(__import__("ctypes").Structure):
    """include/volta_b200_ext.h: vzb_round_job."""

    _C = __import__("ctypes")
    _fields_ = [("kind", _C.c_uint32), ("flags", _C.c_uint32), ("in_id", _C.c_uint64 * 4),
                ("in_offset", _C.c_size_t * 4), ("len", _C.c_size_t), ("r", _C.c_uint64 * 2),
                ("out_id", _C.c_uint64 * 4), ("out_offset", _C.c_size_t * 4), ("s_id", _C.c_uint64),
                ("s_offset", _C.c_size_t), ("msg_id", _C.c_uint64), ("msg_offset", _C.c_size_t),
                ("q_alpha", _C.c_uint64 * 2)]


# DRAM read + write bytes per algorithmic byte of the step-0 replica, from an
# ncu capture of the 2^22-query replica (mean of its 13 launches: 268,123,077 B
# read + 1,230,021 B written for 234,520,576 algorithmic bytes; the parents
# are read at stride 2, so their whole level crosses DRAM)
LOGUP_REPLICA_TRAFFIC = (268123077 + 1230021) / 234520576
# Warp instructions per unit of work of the integer-bound kernels, from ncu
# captures (smsp__inst_executed.sum): the step-0 replica at 2^22 queries
# (42,314,187 for 2,095,104 pairs), the NTT passes at 96 rows x 2^16
# (75,634,080 for 50,331,648 butterflies), the on-chip triple rounds at 2^23
# (197.0 M for 1024 tiles of 8192 entries)
LOGUP_WARP_INST_PER_PAIR = 42314187 / 2095104
NTT_WARP_INST_PER_BUTTERFLY = 75634080 / 50331648
TRIPLE_LOCAL_WARP_INST_PER_TILE = 197.0e6 / 1024
SM_MAX_MHZ = 1965.0  # clocks.max.sm of this pool's B200s


def issue_roofline(warp_instructions: float, ms: float, sm_mhz: float | None = None) -> dict:
    """A kernel's integer-instruction issue rate against the SMs' issue peak
    (4 warp instructions per clock per SM): the roofline of the
    integer-bound Goldilocks kernels, next to their HBM fraction."""
    import torch

    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    mhz = sm_mhz or SM_MAX_MHZ
    peak = sms * 4 * mhz * 1e6
    achieved = warp_instructions / (ms / 1e3)
    return {"bound": "integer instruction issue", "unit": "warp instructions/s", "achieved": round(achieved, 1),
            "peak": round(peak, 1), "frac": round(achieved / peak, 4), "warp_instructions": int(warp_instructions),
            "peak_source": f"4 warp instructions per clock per SM x {sms} SMs x {mhz:.0f} MHz"}


def logup_step0_replica(be, log2_queries: int, reps: int = 10):
    """The proof's largest launch, replicated on seeded data of the same
    shapes: step 0 of the query side's cross-layer round batch, i.e. round 0
    on the interleaved children of every layer with more than 2^11 entries
    per vector (layer L: 2 x 2^L children of P and Q, a 2^(L-1)-entry suffix
    table, and its parent level, whose even entries are the round's t = 0
    terms); the leaf layer's numerators are all 1 and its children are read
    from the 8-byte query column.  Returns (average launch ms, algorithmic
    bytes per launch, jobs)."""
    import ctypes as C

    jobs, bufs, nbytes = [], [], 0
    msg = be.alloc(16 * 4 * 32)
    bufs.append(msg)
    for L in range(min(12, log2_queries - 1), log2_queries):  # at least the leaf layer on small cases
        vlen = 1 << L
        leaf = L == log2_queries - 1
        q = be.alloc((8 if leaf else 16) * 2 * vlen)
        be.call("chacha8_prover_secret_fp_rows_device", q, 0, SUMCHECK_SEED, 100 + L, 1, (2 if leaf else 4) * vlen)
        p = pp = pq = 0
        if not leaf:
            p = be.alloc(16 * 2 * vlen)
            be.call("chacha8_prover_secret_fp_rows_device", p, 0, SUMCHECK_SEED, 200 + L, 1, 4 * vlen)
            pp, pq = be.alloc(16 * vlen), be.alloc(16 * vlen)
            be.call("chacha8_prover_secret_fp_rows_device", pp, 0, SUMCHECK_SEED, 400 + L, 1, 2 * vlen)
            be.call("chacha8_prover_secret_fp_rows_device", pq, 0, SUMCHECK_SEED, 500 + L, 1, 2 * vlen)
        s = be.alloc(16 * (vlen // 2))
        be.call("chacha8_prover_secret_fp_rows_device", s, 0, SUMCHECK_SEED, 300 + L, 1, vlen)
        bufs += [x for x in (p, q, s, pp, pq) if x]
        j = RoundJob()
        # leaf: all-one numerators, children from the query column; else parents given
        j.kind, j.flags, j.len = 0, 3 if leaf else 4, vlen
        j.q_alpha[0], j.q_alpha[1] = 5, 7
        j.in_id[0], j.in_id[1] = p, q
        if not leaf:
            j.out_id[0], j.out_id[1] = pp, pq
        j.s_id, j.msg_id, j.msg_offset = s, msg, 4 * len(jobs)
        jobs.append(j)
        # children (P and Q: 64 B per pair; the leaf column: 16 B), the even
        # parents (2 x 16 B per pair) and the suffix table (16 B per pair)
        nbytes += (16 * vlen if leaf else 64 * vlen + 16 * vlen) + 16 * (vlen // 2)
    arr = (RoundJob * len(jobs))(*jobs)
    call = lambda: be.check(be.lib.volta_b200_logup_round_batch_device(be.ctx, C.cast(arr, C.c_void_p), len(jobs)),
                            "logup_round_batch")  # noqa: E731
    for _ in range(3):
        call()
    be.mark(4)
    for _ in range(reps):
        call()
    be.mark(5)
    ms = be.elapsed_ms(4, 5) / reps
    for x in bufs:
        be.free(x)
    return ms, nbytes, len(jobs)


def config1_leg(args, rank, world, local_rank, dist, prover, peaks, timed_steps=None):
    """BASELINE config 1 through the drop-in ABI: one step = one proof of the
    triple-product sumcheck over three 2^24-entry FpStream tables (24 rounds,
    private-transcript challenges) and the LogUp argument of 2^24 GELU-table
    queries; with N GPUs the one proof is sharded on the top index bits.
    Returns the leg's JSON object (the headline line's shape)."""
    import torch

    from volta_zk_b200 import accel
    from volta_zk_b200.sharded import ShardedProver, concurrently, torch_all_gather, torch_all_to_all

    steps = timed_steps or args.steps
    be = prover.backend
    # lanes = 2: the LogUp proof runs on a second context (its own stream and
    # workspaces) from a second host thread, concurrently with the triple
    # sumcheck, so each protocol's latency-bound stretches overlap the other's work
    prover_b = accel.Prover(policy=1) if args.lanes == 2 else prover
    be_b = prover_b.backend
    n = 1 << args.log2_sumcheck
    n_f, n_t = 1 << args.log2_queries, 1 << args.log2_table
    if world & (world - 1) or n % world or n_f % world or n_t % (2 * world):
        raise SystemExit("the GPU count must be a power of two that divides the tables")

    # ---- inputs resident in HBM (generated on the device through the ABI) ----
    # the tables are Fp values (FpStream rows): kept as Fp columns, proved
    # without lifting them to Fp2 (volta_b200_triple_*_fp rounds)
    tables = []
    for t in range(3):
        col = be.alloc(8 * n)
        be.call("chacha8_prover_secret_fp_rows_device", col, 0, SUMCHECK_SEED, t, 1, n)
        tables.append(col)
    f, table, mult = logup_inputs(args.log2_queries, args.log2_table, accel.fpstream_u64)
    cap = proof_words(n_f, n_t)
    if world == 1:
        shard_tables = tables
        f_col, t_col, m_col = be_b.upload_new(embed_i16(f)), be_b.upload_new(embed_i16(table)), be_b.upload_new(mult)
    else:
        # this rank's slices: entries [rank n / world, (rank + 1) n / world) of every table and column
        nl = n // world
        shard_tables = []
        for tid in tables:
            sl = be.alloc(8 * nl)
            be.call("resident_copy_rows", tid, 8 * nl * rank, 8 * nl, sl, 0, 8 * nl, 1, 8 * nl)
            shard_tables.append(sl)
        fs, ts = slice(rank * n_f // world, (rank + 1) * n_f // world), slice(rank * n_t // world,
                                                                              (rank + 1) * n_t // world)
        f_col = be_b.upload_new(np.ascontiguousarray(embed_i16(f)[fs]))
        t_col = be_b.upload_new(np.ascontiguousarray(embed_i16(table)[ts]))
        m_col = be_b.upload_new(np.ascontiguousarray(mult[ts]))
        dev = torch.device("cuda", local_rank)
        # on two lanes the LogUp lane gathers on its own communicator as soon
        # as its local part is done (every rank creates the group, in order)
        lg_gather = (torch_all_gather(dev, dist.new_group(backend="nccl"))
                     if args.lanes == 2 and args.split_gather else None)
        sharded = ShardedProver(prover, rank, world, torch_all_gather(dev),
                                logup_prover=prover_b if args.lanes == 2 else None, logup_gather=lg_gather)

    def both(run_triple, run_logup):
        """The two protocols of a proof; on two lanes the LogUp part runs in a
        second host thread on the second context."""
        if args.lanes == 1:
            return run_triple(), run_logup()
        return concurrently(run_triple, run_logup)

    def step():
        if world == 1:
            (msgs, finals), proof = both(
                lambda: prover.triple_sumcheck_fp(tables[0], tables[1], tables[2], n, TRANSCRIPT_SEED),
                lambda: prover_b.logup_prove(f_col, n_f, t_col, n_t, m_col, LOGUP_SEED, LOGUP_DOMAIN, cap))
        else:  # local work of both protocols, one all-gather per proof
            msgs, finals, proof = sharded.prove(*shard_tables, n, TRANSCRIPT_SEED, f_col, n_f, t_col, n_t, m_col,
                                                LOGUP_SEED, LOGUP_DOMAIN, base=True)
        return msgs, finals, proof

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    barrier()
    launches0 = be.launches() + (be_b.launches() if be_b is not be else 0)
    with ClockSampler(local_rank) as clocks:
        barrier()
        be.mark(0)
        for _ in range(steps):
            msgs, finals, proof = step()
        be.mark(1)
        ms = be.elapsed_ms(0, 1)
        barrier()
    launches = be.launches() + (be_b.launches() if be_b is not be else 0) - launches0
    step_s = max_over_ranks(ms / 1e3 / steps)

    # ---- e2e through the C ABI with host buffers ---------------------------
    e2e = None
    if not args.no_e2e:
        # The user's inputs in their own formats: the triple tables as Fp
        # columns (8 B per entry), the lookup queries and table as int16
        # witness values (2 B per entry, embedded in Fp on the device), the
        # multiplicities as u32.  The LogUp inputs are uploaded first; the
        # triple columns then stream in by chunks on the first context's copy
        # stream while the LogUp part computes, and each chunk's on-chip
        # triple rounds run as soon as it has landed (HostColumns in the host
        # library).  With N GPUs every rank uploads only its slices.
        nl, nfl, ntl = n // world, n_f // world, n_t // world
        host_cols = [np.ascontiguousarray(be.download(t, 8 * n)[rank * nl:(rank + 1) * nl]) for t in tables]
        pinned = [torch.from_numpy(x.view(np.int64)).pin_memory() for x in host_cols]
        f16_h = torch.from_numpy(np.ascontiguousarray(f[rank * nfl:(rank + 1) * nfl]).astype(np.int16)).pin_memory()
        t16_h = torch.from_numpy(np.ascontiguousarray(table[rank * ntl:(rank + 1) * ntl]).astype(np.int16)).pin_memory()
        mult_h = torch.from_numpy(np.ascontiguousarray(mult[rank * ntl:(rank + 1) * ntl]).astype(np.int32)).pin_memory()
        # the triple tables on the first context, the LogUp inputs on the LogUp lane's
        ups = [be.alloc(8 * nl) for _ in range(3)] + [be_b.alloc(2 * nfl), be_b.alloc(2 * ntl), be_b.alloc(4 * ntl),
                                                      be_b.alloc(8 * nfl), be_b.alloc(8 * ntl)]
        owners = [be] * 3 + [be_b] * 5
        h2d = 3 * 8 * n + 2 * n_f + 2 * n_t + 4 * n_t  # whole job
        d2h = (16 * (3 * args.log2_sumcheck + 3) + 16 * cap) * world
        last = {}

        host_ptrs = [t.data_ptr() for t in pinned]

        def e2e_step():
            for buf, t in zip(ups[3:6], [f16_h, t16_h, mult_h]):
                be_b.upload_async(buf, t.data_ptr(), t.numel() * t.element_size())
            be_b.wait_uploads()
            be_b.embed_i16(ups[3], ups[6], nfl)
            be_b.embed_i16(ups[4], ups[7], ntl)
            # the triple columns stream in from pinned host memory chunk by
            # chunk; each chunk's on-chip rounds run as soon as it has landed
            if world == 1:
                (last["msgs"], last["finals"]), last["proof"] = both(
                    lambda: prover.triple_sumcheck_fp_host(ups[0], ups[1], ups[2], host_ptrs, n, TRANSCRIPT_SEED),
                    lambda: prover_b.logup_prove(ups[6], n_f, ups[7], n_t, ups[5], LOGUP_SEED, LOGUP_DOMAIN, cap))
            else:
                last["msgs"], last["finals"], last["proof"] = sharded.prove(
                    ups[0], ups[1], ups[2], n, TRANSCRIPT_SEED, ups[6], n_f, ups[7], n_t, ups[5], LOGUP_SEED,
                    LOGUP_DOMAIN, base=True, host=host_ptrs)

        e2e_step()
        barrier()
        be.mark(2)
        for _ in range(steps):
            e2e_step()
        be.mark(3)
        e2e_s = max_over_ranks(be.elapsed_ms(2, 3) / 1e3 / steps)
        barrier()
        same = (np.array_equal(last["msgs"], msgs) and np.array_equal(last["finals"], finals)
                and np.array_equal(last["proof"], proof))
        e2e = {"value": e2e_s, "unit": "s/proof", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "inputs": "triple tables as Fp columns, lookup queries and table as int16, multiplicities as u32; "
                         "the triple tables stream in by 16 MiB chunks while the LogUp part and the first 13 "
                         "triple rounds (per landed chunk) compute",
               "proof_matches_resident": bool(same)}
        for owner, b in zip(owners, ups):
            owner.free(b)

    # ---- roofline of the dominant kernel ----------------------------------
    peak = peaks.get("hbm_gbs", 6650.0)
    batch_ms, batch_bytes, batch_jobs = logup_step0_replica(be, args.log2_queries)
    achieved = batch_bytes / (batch_ms / 1e3) / 1e9
    traffic_ratio = LOGUP_REPLICA_TRAFFIC
    roofline = {"bound": "hbm",
                "kernel": f"logup_round_batch_kernel: step 0 of the 2^{args.log2_queries}-query side "
                          f"({batch_jobs} layers in one launch, the proof's largest launch)",
                "achieved": round(achieved, 1), "peak": peak,
                "peak_source": "measured" if "hbm_gbs" in peaks else "fallback", "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": int(batch_bytes * traffic_ratio),
                "traffic_source": "ncu capture of the 2^22-query replica, scaled by algorithmic bytes",
                "algorithmic_bytes": batch_bytes, "avg_launch_ms": round(batch_ms, 4)}
    pairs = sum((1 << L) // 2 for L in range(min(12, args.log2_queries - 1), args.log2_queries))
    roofline["issue"] = issue_roofline(LOGUP_WARP_INST_PER_PAIR * pairs, batch_ms)
    # the triple-product round kernels, at full size (three 2^24 tables)
    mbox = be.alloc(48)
    lifted = [be.alloc(16 * n) for _ in range(3)]
    for col, tid in zip(tables, lifted):
        be.call("base_broadcast_fp2_device", col, 0, tid, 0, n, 1, 2)
    fp_round = be.lib.volta_b200_triple_round_fp_into_device
    # the on-chip pass: rounds 0 .. 12 of the proof's triple sumcheck (both
    # kernels); algorithmic bytes: the three Fp columns read once, plus the
    # round-7 tables (3 x 64 Fp2 per 8192-entry tile) written and read once
    tiles = n // 8192
    loc_r = be.upload_new(np.zeros((13, 2), dtype=np.uint64) + np.uint64(3))
    loc_acc = be.alloc(13 * 12 * 8)
    be.call("resident_zero", loc_acc, 0, 13 * 12 * 8)
    loc_f = [be.alloc(16 * max(tiles, 1)) for _ in range(3)]
    loc_fn = be.lib.volta_b200_triple_local_device
    runs = {}
    if tiles:
        runs[f"triple_local (rounds 0-12 on chip, 2^{args.log2_sumcheck} Fp columns: the proof's triple pass)"] = (
            lambda: be.check(loc_fn(be.ctx, 1, *tables, n, 0, tiles, loc_r, 0, loc_acc, *loc_f), "triple_local"),
            3 * 8 * n + 2 * tiles * 3 * 64 * 16)
    runs |= {
        "triple_round_fp (2^23 pairs, Fp columns: one round of the round-by-round path)":
            (lambda: be.check(fp_round(be.ctx, *tables, n // 2, mbox, 0), "triple_round_fp"), 3 * 8 * n),
        "fp2_triple_product_round (2^23 pairs, Fp2 tables: the reference entry point)":
            (lambda: be.call("fp2_triple_product_round_into_device", lifted[0], 0, lifted[1], 0, lifted[2], 0,
                             n // 2, mbox, 0), 3 * 16 * n),
    }
    kernels = {}
    for name, (call, nbytes) in runs.items():
        for _ in range(3):
            call()
        be.mark(4)
        for _ in range(20):
            call()
        be.mark(5)
        kms = be.elapsed_ms(4, 5) / 20
        kernels[name] = {"avg_launch_ms": round(kms, 4), "algorithmic_bytes": nbytes,
                         "hbm_gbs": round(nbytes / (kms / 1e3) / 1e9, 1),
                         "frac": round(nbytes / (kms / 1e3) / 1e9 / peak, 4)}
        if name.startswith("triple_local"):  # instruction-bound by design: its issue roofline
            kernels[name]["issue"] = issue_roofline(TRIPLE_LOCAL_WARP_INST_PER_TILE * tiles, kms)
    roofline["other_kernels"] = kernels
    for x in lifted + [mbox, loc_r, loc_acc] + loc_f:
        be.free(x)

    cpu, parity = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tabs, logup = cpu_inputs(args.log2_sumcheck, args.log2_queries, args.log2_table)
        ts, threads, ref = cpu_prove_times(tabs, logup, steps=2)
        del tabs
        cpu = {"value": round(min(ts), 4), "unit": "s/proof", "cores": threads, "kind": "port",
               "sample": f"one whole config-1 proof at full size (2^{args.log2_sumcheck} tables, "
                         f"2^{args.log2_queries} queries), best of 2, oracle (C/OpenMP restatement of the reference "
                         "CPU prover)"}
        # the oracle's proof is the checker of the device proof at this size
        parity = bool(np.array_equal(ref[0], msgs) and np.array_equal(ref[1], finals)
                      and np.array_equal(ref[2], proof))
    if prover_b is not prover:
        prover_b.close()
    return {
        "workload": workload_name(args), "value": round(step_s, 6), "unit": "s/proof", "higher_is_better": False,
        "ms_per_step": round(step_s * 1e3, 3), "steps": steps, "scaling": "strong",
        "parallelism": f"one proof sharded over {world} GPU(s) (top index bits; one NCCL all-gather per "
                       f"sumcheck)" if world > 1 else "one proof on one GPU",
        "l2": "inputs larger than L2 (402 MB of Fp tables, 134 MB of queries)",
        "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "gpu_launches": launches, "clocks": clocks.summary(),
        "proof_check": {"parity": parity,
                        "parity_source": "device proof == oracle proof at the measured size" if parity is not None
                        else "not checked in this run (the oracle runs at N = 1); compare sha256 with N = 1",
                        "messages": int(msgs.shape[0]), "proof_words": int(proof.shape[0]),
                        "sha256": hashlib.sha256(np.ascontiguousarray(msgs).tobytes() +
                                                 np.ascontiguousarray(finals).tobytes() +
                                                 np.ascontiguousarray(proof).tobytes()).hexdigest()},
    }


PROOF_SEED, MAC_SEED, PAD_SEED = bytes([0x50] * 32), bytes([0x4D] * 32), bytes([0x11] * 32)


def config3_cpu(t: int, layer: int = 0):
    """The reference's CPU algorithm for config 3 (the oracle restatement:
    oracle/gpt2.py's forward and proof schedule, C/OpenMP primitives, every
    host thread): the whole 12-layer forward at T tokens, the proof of one
    layer (all 12 layers have the same shapes) and the weight commitment,
    each timed.  Returns (timings, the oracle's words of that layer)."""
    from oracle import oracle as o  # checker / baseline only
    from oracle.gpt2 import OracleOps, Schedule, forward_model, pcs_root
    from volta_zk_b200 import gpt2

    o.build()
    threads = o.set_threads(o.host_threads())
    model = gpt2.synthetic_model()
    luts = gpt2.build_luts()
    tokens = gpt2.prefill_tokens(t)
    t0 = time.perf_counter()
    res = forward_model(OracleOps(o), tokens, model, luts, row_shift=1)
    t1 = time.perf_counter()
    words = Schedule(o, luts, t).layer(res["layers"][layer], model.layers[layer], PROOF_SEED, layer)
    t2 = time.perf_counter()
    root = pcs_root(o, model, PAD_SEED)
    t3 = time.perf_counter()
    return {"forward_s": t1 - t0, "layer_s": t2 - t1, "pcs_s": t3 - t2, "threads": threads, "root": root}, words


def plan_split(args, world, layers, costs):
    """gpt2.split_plan, or with --commit unit / rows the commitment forced
    onto one GPU / split by rows (rows needs a power-of-two world)."""
    from volta_zk_b200 import gpt2

    if args.commit == "auto" or world == 1:
        return gpt2.split_plan(world, layers, costs)
    if args.commit == "unit" or world & (world - 1):
        return gpt2.split_sites(world, layers=layers, costs=costs)
    c = costs or (gpt2.LAYER_COST, gpt2.PART_COSTS, gpt2.COMMIT_COST)
    return gpt2.split_sites(world, layers=layers, costs=(c[0], c[1], 0))[0], None


def split_commitment(be, gp, rank, world, dev, pcs_rank):
    """The weight commitment's share of a proof step on this rank: with
    pcs_rank None every rank encodes its row block and the root comes from
    the all-to-all of column chaining values (sharded.gpt2_commit_sharded);
    otherwise the committing rank's prove_units call commits (returns None)."""
    if pcs_rank is not None:
        return lambda: None
    from volta_zk_b200 import sharded

    gather, a2a = sharded.torch_all_gather(dev), sharded.torch_all_to_all(dev)
    return lambda: sharded.gpt2_commit_sharded(be, gp, PAD_SEED, rank, world, gather, a2a)


def commit_note(pcs_rank, world) -> str:
    if pcs_rank is None:
        return (f"the weight commitment split by rows over the {world} GPUs (NCCL all-to-all of the column "
                f"chaining values, all-gather of the slab roots)")
    return f"the weight commitment on rank {pcs_rank}"


def config3(args, rank, world, local_rank, dist, prover, peaks):
    """BASELINE config 3 (the metric): GPT-2 small prefill of T = 1024
    tokens through the drop-in ABI.  One step = the witness forward (embed,
    12 layers, final LN, logits) + the prefill proof schedule over it (per
    layer: 14 LogUp lookup instances, the weight-GEMM, attention and
    LayerNorm/softmax product sumchecks, VOLE-MAC boundary corrections) +
    the Ligero commitment of the weights.  With N GPUs every rank runs the
    forward (replicas) and proves its share: the (layer, site) sub-proofs
    are independent over the same witness, so gpt2.split_plan deals whole
    layers (or layer parts) out by measured costs, largest first onto the
    least-loaded GPU, and gives the commitment to one GPU or splits it by
    rows (an all-to-all of column chaining values) where the cost model
    says that is faster; the words meet in two NCCL all-gathers (word
    counts per site, then the words) and are assembled in layer and site
    order, identical to the one-GPU proof."""
    import torch

    from volta_zk_b200 import gpt2, sharded

    t = args.tokens
    be = prover.backend
    model = gpt2.synthetic_model()
    tokens = gpt2.prefill_tokens(t)
    sess = gpt2.Gpt2Session(prover, model, t)
    sess.forward(tokens)  # uploads the tokens: resident from here on
    gp = gpt2.Gpt2Prover(sess)
    split, pcs_rank = plan_split(args, world, gpt2.LAYERS, None)
    units = split[rank]
    mine = [l for l, m in units if m & (1 << gpt2.SITE_CORRECTIONS)]  # layers whose corrections this rank makes
    dev = torch.device("cuda", local_rank)
    commit = split_commitment(be, gp, rank, world, dev, pcs_rank)

    def step(host_tokens=None):
        sess.forward(host_tokens)
        root = commit()
        words, sites, r = gp.prove_units(PROOF_SEED, MAC_SEED, PAD_SEED, units, rank == pcs_rank)
        return sharded.gather_units(words, sites, split, rank, world, dist, dev, gpt2.LAYERS), None, root or r

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        v = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return float(v.item())

    for _ in range(args.warmup):
        step()
    barrier()
    launches0 = be.launches()
    with ClockSampler(local_rank) as clocks:
        barrier()
        be.mark(0)
        for _ in range(args.steps):
            words, per_layer, root = step()
        be.mark(1)
        ms = be.elapsed_ms(0, 1)
        barrier()
    launches = be.launches() - launches0
    step_s = max_over_ranks(ms / 1e3 / args.steps)
    logits = sess.logits()
    fwd_err = sess.error_word() | max(sess.layer_errors())
    roots = [root]
    if world > 1 and pcs_rank is not None:  # the committing rank's root to every rank
        r = torch.from_numpy(np.frombuffer(root, dtype=np.uint8).copy()).to(dev)
        dist.broadcast(r, pcs_rank)
        roots = [bytes(r.cpu().numpy())]

    # ---- the rho denominator: the plain int16 forward (each rank a replica) --
    reps = max(5, args.steps)
    sess.forward()
    be.mark(4)
    for _ in range(reps):
        sess.forward()
    be.mark(5)
    fwd_s = max_over_ranks(be.elapsed_ms(4, 5) / 1e3 / reps)

    # ---- e2e through the host API with host buffers ----------------------
    e2e = None
    if not args.no_e2e:
        pinned = torch.from_numpy(tokens.view(np.int32)).pin_memory()
        host_tokens = pinned.numpy().view(np.uint32)
        n_corr = len(mine) * 5
        # the boundary corrections land in pinned host memory while the
        # later layers compute (Gpt2Prover::set_correction_sink)
        sink_t = torch.empty(gpt2.LAYERS * 5 * t * gpt2.D, dtype=torch.int64).pin_memory()
        sink = sink_t.numpy().view(np.uint64)
        gp.set_correction_sink(sink)

        def e2e_step():
            out = step(host_tokens)
            if rank == 0:
                sess.logits()
            return out

        e2e_step()
        barrier()
        be.mark(2)
        for _ in range(args.steps):
            ew, _, _ = e2e_step()
        be.mark(3)
        e2e_s = max_over_ranks(be.elapsed_ms(2, 3) / 1e3 / args.steps)
        barrier()
        sink_ok = all(np.array_equal(sink.reshape(gpt2.LAYERS, 5, -1)[l, w], gp.correction(l, w))
                      for l in mine for w in range(5))
        gp.set_correction_sink(None)
        corr_bytes = gpt2.LAYERS * 5 * t * gpt2.D * 8
        e2e = {"value": round(e2e_s, 6), "unit": "s/proof", "h2d_bytes_per_step": 4 * t * world,
               "d2h_bytes_per_step": int(ew.shape[0]) * 16 + 8 * gpt2.VOCAB + 32 + corr_bytes,
               "inputs": "token ids from pinned host memory; out: proof words, PCS root, logits of the last "
                         "position and every boundary correction (the proof's VOLE-MAC payload)",
               "proof_matches_resident": bool(np.array_equal(ew, words)),
               "corrections_downloaded_per_rank": n_corr,
               "corrections": "copied to pinned host memory while the later layers compute; equal to the "
                              f"resident corrections: {sink_ok}"}

    # ---- roofline: the proof's dominant kernel (logup_round_batch_kernel,
    # 42 % of a proof in the launch list): its largest launch shape, step 0
    # of a 2^24-query side's 12 large layers, replicated on seeded data
    peak = peaks.get("hbm_gbs", 6650.0)
    batch_ms, batch_bytes, batch_jobs = logup_step0_replica(be, 24)
    achieved = batch_bytes / (batch_ms / 1e3) / 1e9
    traffic_ratio = LOGUP_REPLICA_TRAFFIC
    roofline = {"bound": "hbm",
                "kernel": f"logup_round_batch_kernel: step 0 of a 2^24-query side ({batch_jobs} layers in one launch, "
                          "the shape of the attention-rectangle lookup instances)",
                "achieved": round(achieved, 1), "peak": peak,
                "peak_source": "measured" if "hbm_gbs" in peaks else "fallback", "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": int(batch_bytes * traffic_ratio),
                "traffic_source": "ncu capture of the 2^22-query replica, scaled by algorithmic bytes",
                "algorithmic_bytes": batch_bytes, "avg_launch_ms": round(batch_ms, 4)}
    pairs = sum((1 << L) // 2 for L in range(12, 24))
    roofline["issue"] = issue_roofline(LOGUP_WARP_INST_PER_PAIR * pairs, batch_ms, clocks.summary().get("sm_mhz"))

    digest = hashlib.sha256(np.ascontiguousarray(words).tobytes() + roots[0]).hexdigest()
    golden = {}
    try:
        g = np.load(os.path.join(ROOT, "tests", "golden", f"gpt2_model_t{t}.npz"))
        golden = {"logits_match_reference_mirror": hashlib.sha256(np.ascontiguousarray(logits).tobytes()).hexdigest()
                  == str(g["logits"])}
    except FileNotFoundError:
        pass
    cpu, parity = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tm, ref_words = config3_cpu(t, 0)
        total = tm["forward_s"] + gpt2.LAYERS * tm["layer_s"] + tm["pcs_s"]
        per_layer_words = ref_words.shape[0]
        parity = bool(np.array_equal(ref_words, words[:per_layer_words]) and tm["root"] == roots[0])
        cpu = {"value": round(total, 3), "unit": "s/proof", "cores": tm["threads"], "kind": "port",
               "sample": f"oracle (C/OpenMP restatement of the reference's CPU algorithm): the whole forward "
                         f"({tm['forward_s']:.2f} s), layer 0's proof ({tm['layer_s']:.2f} s, x 12 identical "
                         f"layers) and the weight commitment ({tm['pcs_s']:.2f} s) at T = {t}"}
    return {
        "metric": METRIC, "value": round(step_s, 6), "unit": "s/proof", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 3), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "int16 witness, Fp2 (u64 Goldilocks) proof",
        "data": "synthetic (rust/volta-gpt2 synthetic_model weights, seed 0x1234; FpStream token ids)",
        "config": {"workload": f"config 3: GPT-2 small prefill proof, T = {t} tokens (witness forward + 12 layer "
                               "proofs + weight commitment)",
                   "model": "gpt2-small (12 layers, d 768, 12 heads, MLP 3072, vocab 50257), int16 fixed point, "
                            "LutParams defaults with the stable softmax",
                   "parallelism": f"forward replicated; the {gpt2.LAYERS} layer proofs (or layer parts) dealt "
                                  f"over {world} GPUs largest first onto the least-loaded GPU; "
                                  f"{commit_note(pcs_rank, world)}; NCCL all-gathers of the per-site word counts "
                                  f"and the words" if world > 1 else "one proof on one GPU",
                   "l2": "working set (witness 1.8 GB, lookup trees, 2.1 GB codeword) far larger than L2",
                   "timing_policy": "wall-only counters"},
        "rho": round(step_s / fwd_s, 2), "forward_s": round(fwd_s, 6),
        "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "gpu_launches": launches, "clocks": clocks.summary(),
        "proof_check": {"parity": parity,
                        "parity_source": "layer 0's words and the weight commitment root == the oracle's at T = "
                                         f"{t}" if parity is not None else
                                         "not checked in this run (the oracle runs at N = 1); compare sha256",
                        "words": int(words.shape[0]), "words_per_layer": int(per_layer_words) if cpu else None,
                        "sha256": digest, "pcs_root": roots[0].hex(), "forward_error_word": int(fwd_err),
                        **golden},
    }


def scaled_leg(args, rank, world, local_rank, dist, prover, steps: int = 3, warmup: int = 2):
    """The scaled synthetic shape of config 4 (24 layers, d_model 1024, 16
    heads of 64, MLP 4096; gpt2.GPT2_SCALED) at a 512-token prefill: the
    witness forward, the 24 layer proofs and the weight commitment (355 M
    weights: 2^15 rows of 2^14), with the same split over N GPUs as config 3
    (replicated forward, layers / layer parts dealt by gpt2.split_plan with
    this shape's measured costs, the commitment on one GPU or split by rows
    with the all-to-all of column chaining values, two NCCL all-gathers of
    the words).  Device-timed, max over ranks."""
    import torch

    from volta_zk_b200 import gpt2, sharded

    t, layers = 512, gpt2.GPT2_SCALED.layers
    be = prover.backend
    dev = torch.device("cuda", local_rank)
    model = gpt2.synthetic_model(shape=gpt2.GPT2_SCALED)
    tokens = gpt2.prefill_tokens(t)
    split, pcs_rank = plan_split(args, world, layers, gpt2.SCALED_COSTS)
    units = split[rank]

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        v = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return float(v.item())

    with gpt2.Gpt2Session(prover, model, t) as sess, gpt2.Gpt2Prover(sess) as gp:
        sess.forward(tokens)
        commit = split_commitment(be, gp, rank, world, dev, pcs_rank)

        def step():
            sess.forward()
            root = commit()
            words, sites, r = gp.prove_units(PROOF_SEED, MAC_SEED, PAD_SEED, units, rank == pcs_rank)
            return sharded.gather_units(words, sites, split, rank, world, dist, dev, layers), root or r

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        be.mark(0)
        for _ in range(steps):
            words, root = step()
        be.mark(1)
        step_s = max_over_ranks(be.elapsed_ms(0, 1) / 1e3 / steps)
        reps = 5
        be.mark(2)
        for _ in range(reps):
            sess.forward()
        be.mark(3)
        fwd_s = max_over_ranks(be.elapsed_ms(2, 3) / 1e3 / reps)
        fwd_err = sess.error_word() | max(sess.layer_errors())
        logits = sess.logits()
        pcs_rows = gp.pcs_rows()
    if world > 1 and pcs_rank is not None:
        r = torch.from_numpy(np.frombuffer(root, dtype=np.uint8).copy()).to(dev)
        dist.broadcast(r, pcs_rank)
        root = bytes(r.cpu().numpy())
    golden = {}
    try:
        g = np.load(os.path.join(ROOT, "tests", "golden", "gpt2_scaled_t512.npz"))
        golden = {"logits_match_reference_mirror": hashlib.sha256(np.ascontiguousarray(logits).tobytes()).hexdigest()
                  == str(g["logits"])}
    except FileNotFoundError:
        pass
    return {"workload": f"config 4, scaled shape: {layers} layers, d_model 1024, 16 heads of 64, MLP 4096, "
                        f"vocab 50257; {t}-token prefill proof (witness forward + {layers} layer proofs + weight "
                        f"commitment of {pcs_rows} x 2^14 weights)",
            "value": round(step_s, 6), "unit": "s/proof", "steps": steps, "warmup": warmup,
            "ms_per_step": round(step_s * 1e3, 3), "rho": round(step_s / fwd_s, 2), "forward_s": round(fwd_s, 6),
            "parallelism": f"forward replicated; layers / layer parts dealt over {world} GPUs; "
                           f"{commit_note(pcs_rank, world)}" if world > 1 else "one proof on one GPU",
            "proof_words": int(words.shape[0]),
            "sha256": hashlib.sha256(np.ascontiguousarray(words).tobytes() + root).hexdigest(),
            "pcs_root": root.hex(), "forward_error_word": int(fwd_err), **golden,
            "note": "parity of this shape's forward, proof, corrections and commitment is pinned against the "
                    "oracle at T = 16 and 100 over 2 layers and for an 8-layer commitment of 16384 rows "
                    "(tests/test_gpu_gpt2_scaled.py); compare sha256 across N"}


def decode_leg(prover, t0: int = 960, n: int = 64, reps: int = 3, curve_chunk: int = 16):
    """Config 4 on one GPU.  Witness: greedy KV-cached decoding of n tokens
    after a t0-token prefill (rust/volta-gpt2/src/decode.rs, the native decode
    baseline of rho_decode) and the band witness of those n rows (band.rs /
    resident.rs band_model_witness_resident) from the full forward over the
    same t0 + n tokens.  Proof: the band's proof as one deferred chunk of n
    rows (block_proof.rs prove_layer_phase1_band, model_proof.rs:2710
    prove_response), rho_decode = band proof / native decode of the n tokens
    (p6_report.rs: (prove_response - prove_prefill) / native decode wall), and
    the flat-cost curve of p6_report.rs:4326-4360: the same n tokens as chunks
    of curve_chunk rows over the growing cache, each proved from the forward
    truncated at its end.  Device-timed."""
    from volta_zk_b200 import gpt2

    be = prover.backend
    model = gpt2.synthetic_model()
    tokens = gpt2.prefill_tokens(t0)
    seed, mac = bytes([0x50] * 32), bytes([0x4D] * 32)
    with gpt2.Gpt2Session(prover, model, t0) as s:
        s.forward(tokens)
        times = []
        for _ in range(reps + 1):  # the first run warms up
            with s.decoder(n) as dec:
                be.mark(0)
                dec.generate(n)
                be.mark(1)
                times.append(be.elapsed_ms(0, 1))
                gen = dec.tokens()
                err = dec.error_word()
        decode_ms = statistics.median(times[1:])
    seq = np.concatenate([tokens, gen]).astype(np.uint32)
    with gpt2.Gpt2Session(prover, model, t0 + n) as s2, gpt2.Gpt2Prover(s2) as gp:
        s2.forward(seq)
        btimes, ptimes = [], []
        for _ in range(reps + 1):
            be.mark(2)
            band = s2.band(t0)
            be.mark(3)
            words, per_layer = gp.prove_band(band, 1, seed, mac)
            be.mark(4)
            btimes.append(be.elapsed_ms(2, 3))
            ptimes.append(be.elapsed_ms(3, 4))
            logits_last = band.logits()[-1]
            band.close()
        full_logits = s2.logits()
    band_prove_ms = statistics.median(ptimes[1:])
    curve = []
    for c in range(n // curve_chunk):
        end = t0 + (c + 1) * curve_chunk
        with gpt2.Gpt2Session(prover, model, end) as sc, gpt2.Gpt2Prover(sc) as gc:
            sc.forward(seq[:end])
            with sc.band(end - curve_chunk) as band:
                gc.prove_band(band, c + 1, seed, mac)  # warm-up
                be.mark(5)
                gc.prove_band(band, c + 1, seed, mac)
                be.mark(6)
                curve.append(round(be.elapsed_ms(5, 6), 3))
    return {"workload": f"config 4: {n} greedy KV-cached decode steps after a {t0}-token prefill "
                        f"(GPT-2 small, 12 layers), the band witness of those {n} rows and its proof "
                        f"as one deferred chunk",
            "decode_ms_per_token": round(decode_ms / n, 4), "decode_tokens_per_s": round(n / (decode_ms / 1e3), 1),
            "band_witness_ms": round(statistics.median(btimes[1:]), 4),
            "band_prove_ms": round(band_prove_ms, 3),
            "band_prove_ms_per_token": round(band_prove_ms / n, 4),
            "rho_decode": round(band_prove_ms / decode_ms, 3),
            "band_proof_words": int(words.shape[0]),
            "band_proof_sha256": hashlib.sha256(words.tobytes()).hexdigest()[:16],
            "flat_cost_curve": {"chunk_rows": curve_chunk, "cache_rows_at_start": [t0 + c * curve_chunk
                                                                                   for c in range(len(curve))],
                                "prove_ms": curve},
            "generated_tokens_sha256": hashlib.sha256(gen.tobytes()).hexdigest()[:16],
            "band_last_logits_equal_full_forward": bool(np.array_equal(logits_last, full_logits)),
            "decode_error_word": int(err),
            "note": "decode is the native baseline (one device launch sequence per token, the next token chosen "
                    "on the device); the band proof's parity is pinned against the oracle's band schedule at "
                    "small sizes (tests/test_gpu_gpt2_proof.py)"}


def run_b200(args, rank, world, local_rank):
    import torch

    from volta_zk_b200 import accel, build_all

    if not os.path.exists(os.path.join(ROOT, "volta_zk_b200", "libvolta_cuda_backend.so")):
        if rank == 0:
            build_all()
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod

        dist_mod.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=120))
        dist = dist_mod
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    prover = accel.Prover(policy=1)  # resident context, wall-only counters (no event overhead)
    be = prover.backend
    if args.workload == "config3":
        line = config3(args, rank, world, local_rank, dist, prover, peaks)
        if not args.no_config1:
            line["config1"] = config1_leg(args, rank, world, local_rank, dist, prover, peaks)
    else:
        c1 = config1_leg(args, rank, world, local_rank, dist, prover, peaks)
        line = {"metric": METRIC, "value": c1["value"], "unit": "s/proof", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": c1["ms_per_step"], "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None, "dtype": "Fp2 (u64 Goldilocks)",
                "data": "synthetic (seeded FpStream tables and GELU-LUT queries)",
                "config": {"workload": c1["workload"], "parallelism": c1["parallelism"], "l2": c1["l2"],
                           "timing_policy": "wall-only counters"},
                **{k: c1[k] for k in ("e2e", "roofline", "cpu_baseline", "gpu_launches", "clocks", "proof_check")}}

    ligero = None
    if not args.no_ligero:
        from volta_zk_b200.sharded import torch_all_gather, torch_all_to_all

        comm = None
        if world > 1:
            dev = torch.device("cuda", local_rank)
            comm = (torch_all_gather(dev), torch_all_to_all(dev))
        ligero = ligero_leg(args, prover, be, peaks, rank, world, comm)
        if world > 1:
            t = torch.tensor([ligero["value"]], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ligero["value"] = round(float(t.item()), 6)

    gemm = None
    if world == 1 and not args.no_gemm:
        gemm = gemm_leg(args, be, peaks)

    ligero_zk = None
    if world == 1 and not args.no_ligero and not args.no_ligero_zk:
        ligero_zk = ligero_zk_leg(prover)

    decode = None
    if world == 1 and args.workload == "config3" and not args.no_decode:
        decode = decode_leg(prover)

    scaled = None
    if args.workload == "config3" and not args.no_scaled:
        scaled = scaled_leg(args, rank, world, local_rank, dist, prover)

    if rank == 0:
        line.update({"ligero": ligero, "ligero_zk": ligero_zk, "witness_gemm": gemm, "config4": decode,
                     "config4_scaled": scaled})
        print(json.dumps(line), flush=True)
    prover.close()
    if dist:
        dist.destroy_process_group()


def workload_name(args) -> str:
    """The config-1 workload both arms name in `config.workload`."""
    return (f"config 1: triple-product sumcheck 3 x 2^{args.log2_sumcheck} Fp2, {args.log2_sumcheck} rounds + "
            f"LogUp 2^{args.log2_queries} queries vs 2^{args.log2_table} table")


def run_reference(args, rank):
    if rank != 0:
        return
    if args.workload == "config3":
        run_reference_config3(args)
        return
    run_reference_config1(args)


def run_reference_config3(args):
    """The reference's CPU algorithm for config 3 (the oracle restatement of
    the forward and the proof schedule, C/OpenMP primitives, every host
    thread).  A whole CPU proof at T = 1024 takes minutes, so each step is
    one layer's share, the sample the B200 arm's workload is made of: layer
    (step mod 12)'s forward from its input plus its proof.  The weight
    commitment and the embedding / final LN / logits are timed once.  value
    = 12 x the mean step + those parts, per proof; ms_per_step is the mean
    step itself (one layer)."""
    from oracle import oracle as o  # the reference arm's CPU algorithm
    from oracle.gpt2 import OracleOps, Schedule, forward_layer, forward_model, pcs_root
    from volta_zk_b200 import gpt2

    o.build()
    threads = o.set_threads(o.host_threads())
    t = args.tokens
    model = gpt2.synthetic_model()
    luts = gpt2.build_luts()
    ops = OracleOps(o)
    tokens = gpt2.prefill_tokens(t)
    t0 = time.perf_counter()
    res = forward_model(ops, tokens, model, luts, row_shift=1)
    whole_forward_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    pcs_root(o, model, PAD_SEED)
    pcs_s = time.perf_counter() - t0
    sch = Schedule(o, luts, t)
    times = []
    for k in range(args.warmup + args.steps):
        layer = k % gpt2.LAYERS
        x = res["layers"][layer]["x_in"]
        t0 = time.perf_counter()
        r = forward_layer(ops, x, model.layers[layer], luts, t, 1)
        sch.layer(r, model.layers[layer], PROOF_SEED, layer)
        times.append(time.perf_counter() - t0)
    layer_s = sum(times[args.warmup:]) / args.steps
    # the forward's parts outside the layers (embed, final LN, logits)
    layer_fwd = []
    for layer in range(min(2, gpt2.LAYERS)):
        t0 = time.perf_counter()
        forward_layer(ops, res["layers"][layer]["x_in"], model.layers[layer], luts, t, 1)
        layer_fwd.append(time.perf_counter() - t0)
    edge_s = max(0.0, whole_forward_s - gpt2.LAYERS * sum(layer_fwd) / len(layer_fwd))
    v = gpt2.LAYERS * layer_s + pcs_s + edge_s
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "s/proof", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(layer_s * 1e3, 2),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "int16 witness, Fp2 (u64 Goldilocks) proof",
            "data": "synthetic (rust/volta-gpt2 synthetic_model weights, seed 0x1234; FpStream token ids)",
            "config": {"workload": f"config 3: GPT-2 small prefill proof, T = {t} tokens (witness forward + 12 layer "
                                   "proofs + weight commitment)",
                       "parallelism": f"the reference's CPU algorithm on {threads} host threads of rank 0"},
            "cpu_baseline": {"value": round(v, 3), "unit": "s/proof", "cores": threads, "kind": "port",
                             "sample": f"each step: one layer's forward + proof at T = {t} (layer = step mod 12; the "
                                       "12 layers have identical shapes); value = 12 x mean step "
                                       f"({layer_s:.3f} s) + weight commitment ({pcs_s:.2f} s) + embed/final LN/"
                                       f"logits ({edge_s:.2f} s), all measured in this run; the Rust reference "
                                       "cannot be built here (no cargo), its CPU algorithm runs as the C/OpenMP "
                                       "oracle restatement"},
            "e2e": {"value": round(v, 3), "unit": "s/proof", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_config1(args):
    """The reference's CPU algorithm (the oracle restatement, all host
    threads) proving the same whole config-1 proof as the B200 arm, every
    step at full size: W untimed proofs, then K timed ones."""
    tabs, logup = cpu_inputs(args.log2_sumcheck, args.log2_queries, args.log2_table)
    ts, threads, _ = cpu_prove_times(tabs, logup, steps=args.warmup + args.steps)
    ts = ts[args.warmup:]
    v = sum(ts) / len(ts)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "s/proof", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v * 1e3, 2), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "Fp2 (u64 Goldilocks)",
            "data": "synthetic (seeded FpStream tables and GELU-LUT queries)",
            "config": {"workload": workload_name(args),
                       "parallelism": f"the reference's CPU algorithm on {threads} host threads of rank 0"},
            "cpu_baseline": {"value": round(v, 4), "unit": "s/proof", "cores": threads, "kind": "port",
                             "sample": "the whole config-1 proof at full size every step (no extrapolation); the "
                                       "Rust reference cannot be built here (no cargo), its CPU algorithm runs as the "
                                       "C/OpenMP oracle restatement"},
            "e2e": {"value": round(v, 4), "unit": "s/proof", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", args.gpus if args.gpus == 1 else 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    run_b200(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
