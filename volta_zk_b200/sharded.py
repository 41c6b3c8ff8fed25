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


def torch_all_gather(device=None, group=None) -> AllGather:
    """All-gather of equally shaped uint64 arrays through torch.distributed
    (NCCL when `device` is a CUDA device, else the process group's backend),
    on `group` (default: the world group)."""
    import torch
    import torch.distributed as dist

    def gather(x: np.ndarray) -> List[np.ndarray]:
        t = torch.from_numpy(np.ascontiguousarray(x).view(np.int64).reshape(-1))
        if device is not None:
            t = t.to(device)
        world = dist.get_world_size(group)
        out = torch.empty(world * t.numel(), dtype=torch.int64, device=t.device)
        dist.all_gather_into_tensor(out, t, group=group)
        parts = out.cpu().numpy().view(np.uint64).reshape(world, -1)
        return [p.reshape(x.shape) for p in parts]

    return gather


_LANES = {}


def _lane(device):
    """One persistent worker thread per CUDA device (created on first use,
    bound to the device once), so a proof does not pay for a thread start."""
    ex = _LANES.get(device)
    if ex is None:
        from concurrent.futures import ThreadPoolExecutor

        def bind():
            if device is not None:
                import torch

                torch.cuda.set_device(device)

        ex = ThreadPoolExecutor(max_workers=1, initializer=bind, thread_name_prefix="volta-lane")
        _LANES[device] = ex
    return ex


def concurrently(first, second):
    """Run `second` on this device's lane thread while `first` runs in this
    one (the library's calls release the GIL); both results, or the first
    error.  The lane thread runs on this thread's current CUDA device (a new
    thread starts on device 0, where another GPU's contexts are invalid)."""
    device = None
    try:
        import torch

        if torch.cuda.is_available():
            device = torch.cuda.current_device()
    except ImportError:
        pass
    fut = _lane(device).submit(second)
    try:
        a = first()
    finally:
        err = fut.exception()  # waits for `second` whatever `first` did
    if err is not None:
        raise err
    return a, fut.result()


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

    def __init__(self, prover, rank: int, world: int, all_gather: AllGather, logup_prover=None,
                 logup_gather: AllGather = None):
        """logup_prover: a second Prover (its own context) on which prove()
        runs the LogUp part concurrently with the triple part.  logup_gather:
        an all-gather on a second communicator; with it, the LogUp lane
        gathers and finishes its proof as soon as its local part is done
        (under the triple part's upload or compute) instead of joining the
        triple part's gather."""
        if world & (world - 1):
            raise ValueError("the shard count must be a power of two")
        self.prover, self.rank, self.world, self.gather = prover, rank, world, all_gather
        self.logup_prover = logup_prover
        self.logup_gather = logup_gather
        self.s = world.bit_length() - 1

    def triple_sumcheck(self, a: int, b: int, c: int, n: int, seed: bytes, base: bool = False):
        """a, b, c: this shard's slices (n / world entries) of the tables;
        base: they are Fp columns (tables whose c1 is 0) rather than Fp2."""
        local = self.prover.triple_sumcheck_fp if base else self.prover.triple_sumcheck
        msgs, finals = local(a, b, c, n // self.world, seed)
        parts = self.gather(np.concatenate([msgs, finals]).astype(np.uint64))
        return triple_finish(parts, n, seed)

    def prove(self, a: int, b: int, c: int, n: int, triple_seed: bytes, f_col: int, n_f: int, t_col: int, n_t: int,
              mult: int, logup_seed: bytes, domain: int, base: bool = False, host=None, chunk: int = 0):
        """Both parts of a config-1 proof with one local call and one
        all-gather (two, on two communicators, with logup_gather): (triple
        messages, triple finals, LogUp proof words), equal to triple_sumcheck
        followed by logup_prove.  `host`: this shard's
        triple columns (base only) still in pinned host memory, three
        addresses; they fill a, b, c chunk by chunk under the first rounds."""
        nl = n // self.world
        if self.logup_prover is None:
            local = self.prover.proof_local(a, b, c, nl, base, triple_seed, f_col, n_f // self.world, t_col,
                                            n_t // self.world, mult, self.s, logup_seed, domain, host, chunk)
        else:
            def triple_part():
                if host is not None:
                    m, f = self.prover.triple_sumcheck_fp_host(a, b, c, host, nl, triple_seed, chunk)
                    return np.concatenate([m, f])
                self.prover.backend.wait_uploads()  # tables still arriving on the copy stream, if any
                local_sumcheck = self.prover.triple_sumcheck_fp if base else self.prover.triple_sumcheck
                m, f = local_sumcheck(a, b, c, nl, triple_seed)
                return np.concatenate([m, f])

            def logup_part():
                local = self.logup_prover.logup_local(f_col, n_f // self.world, t_col, n_t // self.world, mult,
                                                      self.s, logup_seed, domain)
                if self.logup_gather is None:
                    return local
                # its own communicator: no ordering against the triple gather
                return logup_finish(self.logup_gather(local), n_f, n_t, logup_seed, domain)

            tri, lg = concurrently(triple_part, logup_part)
            if self.logup_gather is not None:
                msgs, finals = triple_finish(self.gather(tri), n, triple_seed)
                return msgs, finals, lg
            local = np.concatenate([tri, lg])
        parts = self.gather(local)
        kt = 3 * (nl.bit_length() - 1) + 3
        msgs, finals = triple_finish([p[:kt] for p in parts], n, triple_seed)
        proof = logup_finish([p[kt:] for p in parts], n_f, n_t, logup_seed, domain)
        return msgs, finals, proof

    def logup_prove(self, f_col: int, n_f: int, t_col: int, n_t: int, mult: int, seed: bytes, domain: int):
        """f_col / t_col / mult: this shard's slices of the global columns."""
        local = self.prover.logup_local(f_col, n_f // self.world, t_col, n_t // self.world, mult, self.s, seed,
                                        domain)
        return logup_finish(self.gather(local), n_f, n_t, seed, domain)


# ---------------------------------------------------------------------------
# Ligero commitment over G GPUs (rust/volta-pcs/src/ligero.rs:465-505 commit,
# 1440-1480 openings).  Shard g encodes rows [g R/G, (g+1) R/G): its ChaCha8
# message rows, zero padding and row NTTs are local.  A column's BLAKE3 tree
# over R = 128 * 2^k rows is a perfect tree of 1 KiB chunks, so shard g's rows
# are one aligned subtree of it: the shard hashes each column's subtree to a
# 32-byte chaining value, and one all-to-all hands shard s the values of its
# slab of code_len / G columns.  Shard s merges them into its column leaves,
# builds the Merkle subtree of its slab and all-gathers its slab root; the
# top log2 G levels are hashed on one device from the G roots.  Openings: each
# shard gathers its rows of the queried columns and the paths inside its slab.
# ---------------------------------------------------------------------------

H = 32  # bytes per hash


def ligero_shard_encode(be, row_seed: bytes, row0: int, rows_local: int, msg_len: int, code_len: int):
    """Phase 1 (per shard): resident codeword rows and their column chaining
    values (numpy [code_len, 32] uint8)."""
    msgs = be.alloc(8 * rows_local * msg_len)
    be.call("chacha8_prover_secret_fp_rows_device", msgs, 0, row_seed, row0, rows_local, msg_len)
    code = be.alloc(8 * rows_local * code_len)
    if msg_len < code_len:
        be.call("resident_zero", code, 0, 8 * rows_local * code_len)
    be.call("resident_copy_rows", msgs, 0, 8 * msg_len, code, 0, 8 * code_len, rows_local, 8 * msg_len)
    be.free(msgs)
    be.call("ntt_fp_batch_device", code, 0, rows_local, code_len, code, 0)
    cvs = be.alloc(H * code_len)
    be.check(be.lib.volta_b200_hash_fp_column_cvs_device(be.ctx, code, 0, rows_local, code_len, row0 // 128, cvs, 0),
             "hash_fp_column_cvs_device")
    host = be.download(cvs, H * code_len, dtype=np.uint8).reshape(code_len, H)
    be.free(cvs)
    return code, host


def ligero_shard_tree(be, recv: np.ndarray, shards: int, slab: int):
    """Phase 2 (per shard): the Merkle tree of this shard's column slab from
    the received chaining values ([shards, slab, 32]); returns (tree id, slab
    root bytes)."""
    buf = be.upload_new(np.ascontiguousarray(recv, dtype=np.uint8))
    tree = be.alloc(H * (2 * slab - 1))
    be.check(be.lib.volta_b200_merkle_from_cvs_device(be.ctx, buf, 0, shards, slab, tree, 0), "merkle_from_cvs_device")
    be.free(buf)
    root = be.download(tree, H, dtype=np.uint8, offset_bytes=H * (2 * slab - 2))
    return tree, root


def ligero_top_tree(be, roots: np.ndarray) -> np.ndarray:
    """The Merkle levels above the G slab roots ([G, 32]): full top tree
    [(2G - 1), 32], global root last."""
    G = roots.shape[0]
    tree = be.alloc(H * (2 * G - 1))
    be.upload(tree, np.ascontiguousarray(roots, dtype=np.uint8))
    be.check(be.lib.volta_b200_merkle_levels_device(be.ctx, tree, 0, G), "merkle_levels_device")
    out = be.download(tree, H * (2 * G - 1), dtype=np.uint8).reshape(2 * G - 1, H)
    be.free(tree)
    return out


def ligero_shard_open(be, code: int, rows_local: int, code_len: int, tree: int, slab: int, shard: int,
                      idx: np.ndarray):
    """Phase 3 (per shard): this shard's rows of the queried columns
    ([q, rows_local]) and, for the queries inside its slab, their paths up to
    the slab root ([q, log2 slab, 32]; zeros for other queries)."""
    q = idx.size
    ids = be.upload_new(idx.astype(np.uint32))
    cols = be.alloc(8 * q * rows_local)
    be.call("pcs_gather_columns_device", code, 0, rows_local, code_len, ids, 0, q, cols, 0, 0)
    columns = be.download(cols, 8 * q * rows_local).reshape(q, rows_local)
    bits = slab.bit_length() - 1
    local = np.where(idx // slab == shard, idx % slab, slab).astype(np.uint32)  # out of range -> zero path
    paths = np.zeros((q, bits, H), dtype=np.uint8)
    if bits:
        lid = be.upload_new(local)
        pid = be.alloc(H * q * bits)
        be.call("merkle_paths_device", tree, 0, slab, lid, 0, q, pid, 0)
        paths = be.download(pid, H * q * bits, dtype=np.uint8).reshape(q, bits, H)
        be.free(lid)
        be.free(pid)
    be.free(ids)
    be.free(cols)
    return columns, paths


def ligero_assemble(parts_cols, parts_paths, top: np.ndarray, idx: np.ndarray, slab: int):
    """Openings from every shard's phase-3 output and the top tree: columns
    [q, R] (rows in shard order) and full paths [q, log2 code_len, 32]."""
    G = len(parts_cols)
    columns = np.concatenate(parts_cols, axis=1)
    owner = idx // slab
    local = np.stack([parts_paths[int(o)][k] for k, o in enumerate(owner)])
    top_bits = G.bit_length() - 1
    top_paths = np.zeros((idx.size, top_bits, H), dtype=np.uint8)
    for k, o in enumerate(owner):
        node, off, width = int(o), 0, G
        for lv in range(top_bits):
            top_paths[k, lv] = top[off + (node ^ 1)]
            off += width
            width //= 2
            node >>= 1
    return columns, np.concatenate([local, top_paths], axis=1)


def ligero_query_indices(chal_seed: bytes, queries: int, code_len: int) -> np.ndarray:
    """challenge_fp2().c0 mod code_len from FpStream(seed, u64::MAX) (ligero.rs:1444)."""
    from .accel import fpstream_fp2

    return (fpstream_fp2(chal_seed, 2**64 - 1, queries)[:, 0] % np.uint64(code_len)).astype(np.uint32)


def torch_all_to_all(device=None):
    """All-to-all of uint8 arrays [G, ...]: block s goes to rank s; returns
    the blocks received from every rank, in rank order."""
    import torch
    import torch.distributed as dist

    def exchange(x: np.ndarray) -> np.ndarray:
        t = torch.from_numpy(np.ascontiguousarray(x).reshape(-1))
        if device is not None:
            t = t.to(device)
        out = torch.empty_like(t)
        dist.all_to_all_single(out, t)
        return out.cpu().numpy().reshape(x.shape)

    return exchange


def ligero_commit_open_sharded(be, rank: int, world: int, all_gather: AllGather, all_to_all, row_seed: bytes,
                               rows: int, msg_len: int, code_len: int, queries: int, chal_seed: bytes):
    """One Ligero commitment + openings over `world` GPUs; every rank returns
    (root bytes, indices, columns [q, rows], paths [q, log2 code_len, 32]),
    equal to the one-GPU result."""
    if rows % (128 * world) or (rows // 128) & (rows // 128 - 1) or code_len % world:
        raise ValueError("sharded Ligero needs rows = 128 * 2^k divisible by 128 * world")
    rl, slab = rows // world, code_len // world
    code, cvs = ligero_shard_encode(be, row_seed, rank * rl, rl, msg_len, code_len)
    recv = all_to_all(cvs.reshape(world, slab, H))
    tree, root = ligero_shard_tree(be, recv, world, slab)
    roots = np.stack(all_gather(np.frombuffer(root.tobytes(), dtype=np.uint64).copy()))
    top = ligero_top_tree(be, roots.view(np.uint8).reshape(world, H))
    idx = ligero_query_indices(chal_seed, queries, code_len)
    cols, paths = ligero_shard_open(be, code, rl, code_len, tree, slab, rank, idx)
    all_cols = all_gather(cols)
    all_paths = [p.view(np.uint8).reshape(paths.shape)
                 for p in all_gather(np.ascontiguousarray(paths).view(np.uint64))]
    be.free(code)
    be.free(tree)
    columns, full_paths = ligero_assemble(all_cols, all_paths, top, idx, slab)
    return top[-1].tobytes(), idx, columns, full_paths


def gather_units(words, sites, split, rank, world, dist, dev, layers):
    """Every rank's GPT-2 proof words (Gpt2Prover.prove_units over its units
    split[rank]) -> the whole proof in layer and site order, on every rank:
    one all-gather of the word counts per (layer, site)
    (0 where another rank proves it), one of the words (padded to the
    longest rank), then gpt2.assemble_units."""
    import torch

    from . import gpt2

    if world == 1:
        return words
    counts = np.zeros((layers, 25), np.int64)
    for (layer, _), us in zip(split[rank], sites):
        for site, n in us:
            counts[layer, site] = n
    # outputs concatenated along dim 0 (the form every backend takes)
    c = torch.from_numpy(counts).to(dev)
    call = torch.empty((world * layers, 25), dtype=c.dtype, device=dev)
    dist.all_gather_into_tensor(call, c)
    counts_all = call.cpu().numpy().reshape(world, layers, 25)
    totals = counts_all.reshape(world, -1).sum(axis=1)
    longest = int(totals.max())
    buf = np.zeros((longest, 2), dtype=np.uint64)
    buf[:words.shape[0]] = words
    src = torch.from_numpy(buf.view(np.int64)).to(dev)
    out = torch.empty((world * longest, 2), dtype=src.dtype, device=dev)
    dist.all_gather_into_tensor(out, src)
    allw = out.cpu().numpy().view(np.uint64).reshape(world, longest, 2)
    pieces = []
    for g in range(world):
        sites_g = [[(k, int(counts_all[g, l, k])) for k in gpt2.SITE_ORDER if (m >> k) & 1] for l, m in split[g]]
        pieces.append((split[g], allw[g, :int(totals[g])], sites_g))
    return gpt2.assemble_units(pieces, layers=layers)


def gpt2_commit_sharded(be, gp, pad_seed: bytes, rank: int, world: int, all_gather: AllGather, all_to_all) -> bytes:
    """The GPT-2 weight commitment (Gpt2Prover's Ligero matrix: pcs_rows x
    2^14 int16 + 512 ChaCha8 pads per row, RS code 2^15, BLAKE3 column tree)
    over `world` GPUs by rows, like ligero_commit_open_sharded: rank g
    encodes rows g * R / G .. (g + 1) * R / G - 1 and hashes their column
    chaining values (Gpt2Prover.commit_rows), one all-to-all hands every rank
    its column slab's values from all row blocks, each rank builds its slab
    subtree, and the G slab roots meet in an all-gather for the top levels.
    Every rank returns the root, equal to the one-GPU commitment's."""
    rows, code_len = gp.pcs_rows(), 1 << 15
    rl, slab = rows // world, code_len // world
    if rows % (128 * world) or (rl // 128) & (rl // 128 - 1) or code_len % world:
        raise ValueError("sharded weight commitment needs rows / world = 128 * 2^k")
    cvs = gp.commit_rows(pad_seed, rank * rl, rl)
    recv = all_to_all(cvs.reshape(world, slab, H))
    tree, root = ligero_shard_tree(be, recv, world, slab)
    be.free(tree)
    roots = np.stack(all_gather(np.frombuffer(root.tobytes(), dtype=np.uint64).copy()))
    top = ligero_top_tree(be, roots.view(np.uint8).reshape(world, H))
    return top[-1].tobytes()


# ---------------------------------------------------------------------------
# VOLE-MAC epilogue rows over G GPUs.  Row i of an authenticated tensor draws
# its masks from its own correlation domain (tag << 32) | i
# (rust/volta-gpt2/src/gemm.rs:120-154; corr.rs:234-255), so a row block is
# independent work: shard g expands the masks of its rows on its GPU and runs
# the fused GEMM epilogue on its block of A with the whole B.  Nothing is
# exchanged; the blocks concatenate to the single-GPU output and corrections.
# ---------------------------------------------------------------------------

def row_block(m: int, rank: int, world: int):
    """(first row, rows) of shard `rank`: contiguous blocks, the first m % world
    one row longer."""
    if world < 1 or not 0 <= rank < world:
        raise AccelError(f"invalid shard {rank} of {world}")
    base, extra = divmod(m, world)
    row0 = rank * base + min(rank, extra)
    return row0, base + (1 if rank < extra else 0)


def auth_gemm_rows_shard(be, rank: int, world: int, a_id: int, b_id: int, m: int, k: int, n: int, shift: int,
                         mac_seed: bytes, tag: int):
    """This shard's rows of out = requant(A B) and its corrections out - mask
    (volta_cuda_gemm_requant_auth_device on rows [row0, row0 + rows) of the
    resident i16 A (m x k) and the resident B (k x n)).  Returns (row0, rows,
    out id (i16), correction id (u64)); ids are 0 for an empty block."""
    if not 0 <= tag < (1 << 29):
        raise AccelError("tensor tag must leave the reserved domain bits clear")
    row0, rows = row_block(m, rank, world)
    if rows == 0:
        return row0, 0, 0, 0
    masks = be.alloc(8 * rows * n)
    out, corr = be.alloc(2 * rows * n), be.alloc(8 * rows * n)
    try:
        be.call("mock_correlation_sub_masks_device", masks, 0, mac_seed, (tag << 32) | row0, rows, n)
        be.call("gemm_requant_auth_device", a_id, row0 * k, b_id, 0, masks, 0, out, 0, corr, 0, rows, k, n,
                shift)
    except Exception:
        be.free(out)
        be.free(corr)
        raise
    finally:
        be.free(masks)
    return row0, rows, out, corr
