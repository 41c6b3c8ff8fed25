"""One proof over G = 2^s GPUs (one process per GPU, torch.distributed).

Every table of the triple-product sumcheck and every fraction-tree side of
LogUp is split into G contiguous slices; shard g owns the slice whose top
log2 G index bits equal g.  Variables are folded LSB-first
(rust/volta-proto/src/mle.rs:1-30), so the first k - s rounds of a k-variable
sumcheck only pair entries inside one slice: each shard runs them on its own
GPU and its round accumulators are its share of the global ones.  In the clear
sink / private transcript every challenge is a seeded stream draw that never
absorbs a message (logup.rs:1601-1622, transcript.rs:84-103), so all local
rounds of every layer run first and the shards then exchange, once per
proof, their round accumulators, their subtree roots and the few values left
after their local rounds (one all-gather of a few KB).  The last s rounds of
each sumcheck and the top s levels of each fraction tree (2^s entries) are
finished on the host (libvolta_accel: sharded.cpp) with exact field
arithmetic.  The result is the single-GPU proof word for word.

LogUp shares are scaled per layer by eq(top coordinates of the claim point,
g): shard g computes its suffix-eq tables from the truncated point, which
equals the global table restricted to its slice up to that factor.
"""

from __future__ import annotations

import ctypes as C
from typing import Callable, List, Sequence

import numpy as np

from .accel import AccelError, _ptr, load_host_library

AllGather = Callable[[np.ndarray], List[np.ndarray]]


def torch_all_gather(device=None) -> AllGather:
    """All-gather of equally shaped uint64 arrays through torch.distributed
    (NCCL when `device` is a CUDA device, else the process group's backend)."""
    import torch
    import torch.distributed as dist

    def gather(x: np.ndarray) -> List[np.ndarray]:
        t = torch.from_numpy(np.ascontiguousarray(x).view(np.int64).reshape(-1))
        if device is not None:
            t = t.to(device)
        out = torch.empty(dist.get_world_size() * t.numel(), dtype=torch.int64, device=t.device)
        dist.all_gather_into_tensor(out, t)
        parts = out.cpu().numpy().view(np.uint64).reshape(dist.get_world_size(), -1)
        return [p.reshape(x.shape) for p in parts]

    return gather


def _host():
    L = load_host_library()
    if not getattr(L, "_sharded_declared", False):
        vp, sz, u64 = C.c_void_p, C.c_size_t, C.c_uint64
        L.vzh_triple_finish.argtypes = [vp, sz, sz, C.c_char_p, vp, vp, C.c_char_p, sz]
        L.vzh_logup_finish.argtypes = [vp, sz, sz, sz, sz, C.c_char_p, u64, vp, sz, C.POINTER(C.c_size_t),
                                       C.c_char_p, sz]
        L._sharded_declared = True
    return L


def triple_finish(parts: Sequence[np.ndarray], n: int, seed: bytes):
    """Global (messages [k x 3], finals [3]) from every shard's
    concatenated (messages of its own rounds, its 3 final values)."""
    flat = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.uint64).reshape(-1, 2) for p in parts]))
    k = n.bit_length() - 1
    msgs = np.zeros((3 * k, 2), dtype=np.uint64)
    finals = np.zeros((3, 2), dtype=np.uint64)
    err = C.create_string_buffer(1024)
    if _host().vzh_triple_finish(_ptr(flat), len(parts), n, seed, _ptr(msgs), _ptr(finals), err, 1024):
        raise AccelError(err.value.decode())
    return msgs, finals


def logup_finish(parts: Sequence[np.ndarray], n_f: int, n_t: int, seed: bytes, domain: int) -> np.ndarray:
    """The global LogUp proof words from every shard's vzh_logup_local words."""
    per = parts[0].shape[0]
    flat = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.uint64).reshape(-1, 2) for p in parts]))

    def side(n):
        d = n.bit_length() - 1
        return 2 + sum(2 * l + 4 for l in range(d))

    cap = 1 + side(n_f) + side(n_t)
    out = np.zeros((cap, 2), dtype=np.uint64)
    written = C.c_size_t()
    err = C.create_string_buffer(1024)
    if _host().vzh_logup_finish(_ptr(flat), len(parts), per, n_f, n_t, seed, domain, _ptr(out), cap,
                                C.byref(written), err, 1024):
        raise AccelError(err.value.decode())
    return out[: written.value]


class ShardedProver:
    """Runs this shard's local work on its GPU through a Prover (the host
    mirror over the seam) and completes the proof after one all-gather."""

    def __init__(self, prover, rank: int, world: int, all_gather: AllGather):
        if world & (world - 1):
            raise ValueError("the shard count must be a power of two")
        self.prover, self.rank, self.world, self.gather = prover, rank, world, all_gather
        self.s = world.bit_length() - 1

    def triple_sumcheck(self, a: int, b: int, c: int, n: int, seed: bytes):
        """a, b, c: this shard's slices (n / world entries) of the tables."""
        msgs, finals = self.prover.triple_sumcheck(a, b, c, n // self.world, seed)
        parts = self.gather(np.concatenate([msgs, finals]).astype(np.uint64))
        return triple_finish(parts, n, seed)

    def logup_prove(self, f_col: int, n_f: int, t_col: int, n_t: int, mult: int, seed: bytes, domain: int):
        """f_col / t_col / mult: this shard's slices of the global columns."""
        local = self.prover.logup_local(f_col, n_f // self.world, t_col, n_t // self.world, mult, self.s, seed,
                                        domain)
        return logup_finish(self.gather(local), n_f, n_t, seed, domain)
