"""Transcript binding and proof wire format of the blind LogUp argument, on
the CPU: the host library's BLAKE3 (hash and derive-key modes) and the
oracle's against the pinned `blake3` module; the transcript's canonical move
encoding (rust/volta-mac/src/transcript.rs:215-233, 362-380, 654-667) built
by hand; the BlindLogupProof wire bytes (model_proof_codec.rs rules) of the
oracle's blind prover decoded strictly by the host library, and mutated
encodings rejected."""

import numpy as np
import pytest

from oracle import blind as ob

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.usefixtures("package_built")
CTX = "volta-zk/transcript/canonical-moves/v1"


@pytest.mark.parametrize("n", [0, 1, 63, 64, 65, 1023, 1024, 1025, 2048, 3073, 65536 + 7])
def test_blake3_modes_match_the_pinned_crate(oracle, n):
    blake3 = pytest.importorskip("blake3")
    from volta_zk_b200 import accel

    data = bytes((i * 31 + 7) % 256 for i in range(n))
    assert accel.blake3(data) == blake3.blake3(data).digest()
    for ctx in (CTX, "x", ""):
        exp = blake3.blake3(data, derive_key_context=ctx).digest()
        assert accel.blake3(data, ctx) == exp
        assert oracle.blake3_derive_key(ctx, data) == exp


def test_transcript_move_encoding(oracle):
    blake3 = pytest.importorskip("blake3")
    tx = ob.Transcript(oracle, bytes([9] * 32))
    tx.append_fp2s("logup_root_corrections", [(1, 2), (P - 1, 0)])
    c = tx.challenge_fp2()
    assert c == oracle.FpStream(bytes([9] * 32), (1 << 64) - 1).next_fp2()
    label = b"logup_root_corrections"
    msg = (1).to_bytes(8, "little") + (2).to_bytes(8, "little") + (P - 1).to_bytes(8, "little") + bytes(8)
    moves = bytes([1]) + len(label).to_bytes(2, "little") + label + len(msg).to_bytes(8, "little") + msg + bytes([3, 2])
    assert bytes(tx.moves) == moves
    assert tx.digest() == blake3.blake3(moves, derive_key_context=CTX).digest()
    assert tx.ledger == {"logup_root_corrections": 32}


def _case(log2f, log2t, seed):
    rng = np.random.default_rng(seed)
    nf, nt = 1 << log2f, 1 << log2t
    table = rng.integers(-32768, 32768, size=nt).astype(np.int16)
    idx = rng.integers(0, nt, size=nf)
    return table[idx], table, np.bincount(idx, minlength=nt).astype(np.uint32)


@pytest.mark.parametrize("log2f,log2t", [(1, 1), (4, 3), (9, 6)])
def test_blind_logup_wire_bytes_decode_strictly(oracle, log2f, log2t):
    from volta_zk_b200 import accel

    f, table, mult = _case(log2f, log2t, log2f * 10 + log2t)
    data, digest, tx_bytes, dom = ob.blind_logup_prove(oracle, f, table, mult, bytes([0x5A] * 32),
                                                       bytes([0x4D] * 32), 0x700)
    rounds = accel.blind_logup_check(data)
    assert rounds == list(range(log2f)) + list(range(log2t))
    # BlindLogupProof::bytes (logup.rs:1877-1884, 3171-3174) is the transcript's charge
    frac = lambda d: 32 + sum(16 * (2 * r + 7) for r in range(d))  # noqa: E731
    assert tx_bytes == frac(log2f) + frac(log2t) + 64
    # one domain per root, round, split, product group, plus the cross group
    assert dom - 0x700 == sum(1 + sum(r + 2 for r in range(d)) for d in (log2f, log2t)) + 1
    bad = bytearray(data)
    bad[8:16] = (P).to_bytes(8, "little")  # root correction c1 = p: not canonical
    with pytest.raises(accel.AccelError, match="noncanonical"):
        accel.blind_logup_check(bytes(bad))
    with pytest.raises(accel.AccelError, match="trailing"):
        accel.blind_logup_check(data + b"\x00")
    with pytest.raises(accel.AccelError, match="truncated"):
        accel.blind_logup_check(data[:-1])
    at = 32 + 4 + sum(4 + 32 * r + 112 for r in range(log2f))  # the lookup side's aux tag
    bad = bytearray(data)
    bad[at] = 2
    with pytest.raises(accel.AccelError, match="option tag"):
        accel.blind_logup_check(bytes(bad))
    bad = bytearray(data)
    bad[32:36] = (1000001).to_bytes(4, "little")
    with pytest.raises(accel.AccelError, match="strict cap"):
        accel.blind_logup_check(bytes(bad))
