"""CPU checks of the drop-in boundary: the library builds, loads, exports
exactly the symbols include/volta_cuda_backend.h declares (the set the
reference's Rust loader resolves eagerly, rust/volta-accel/src/cuda.rs:
1159-1420), reports ABI 37, and fails loudly without a device."""

import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def built():
    from volta_zk_b200 import build_all

    build_all()
    return True


def exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True)
    return {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}


def test_header_declares_124_symbols():
    from volta_zk_b200 import accel

    decls = accel.parse_header()
    assert len(decls) == 124
    assert all(n.startswith("volta_cuda_") for n in decls)


def test_library_exports_exactly_the_header(built):
    from volta_zk_b200 import accel

    syms = exported(os.path.join(ROOT, "volta_zk_b200", "libvolta_cuda_backend.so"))
    cuda_syms = {s for s in syms if s.startswith("volta_cuda_")}
    assert cuda_syms == set(accel.parse_header())
    ext = set(re.findall(r"\b(volta_b200_\w+)\(", open(os.path.join(ROOT, "include", "volta_b200_ext.h")).read()))
    assert syms == cuda_syms | ext, "nothing but the C ABI and its declared extensions is exported"


def test_loader_checks_version_and_symbols(built):
    from volta_zk_b200 import accel

    lib = accel.load_cuda_library()
    assert lib.volta_cuda_abi_version() == 37


def test_host_library_exports(built):
    syms = exported(os.path.join(ROOT, "volta_zk_b200", "libvolta_accel.so"))
    for name in ("vzh_open", "vzh_close", "vzh_triple_sumcheck", "vzh_logup_prove", "vzh_stats"):
        assert name in syms


def test_struct_layouts():
    from volta_zk_b200 import accel

    assert C.sizeof(accel.RawStats) == 504
    assert C.sizeof(accel.Fp2) == 16


def test_missing_library_fails_loudly(tmp_path):
    from volta_zk_b200 import accel

    with pytest.raises(accel.AccelError, match="LibraryLoad"):
        accel.load_cuda_library(str(tmp_path / "nope.so"))


def test_no_device_fails_loudly(built):
    """Requesting CUDA on a host without a device is an error, never a CPU
    fallback (rust/volta-accel/src/lib.rs:1038-1044)."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from volta_zk_b200 import accel

    with pytest.raises(accel.AccelError, match="Cuda:"):
        accel.CudaBackend()
    with pytest.raises(accel.AccelError):
        accel.Prover()


def test_header_compiles_as_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "volta_cuda_backend.h"\n'
                   '_Static_assert(sizeof(vz_raw_stats) == 504, "stats");\n'
                   '_Static_assert(sizeof(vz_raw_pinned_stats) == 104, "pinned");\n'
                   '_Static_assert(sizeof(vz_raw_control_state) == 104, "control");\n'
                   '_Static_assert(sizeof(vz_fp2) == 16, "fp2");\n'
                   'int main(void) { return (int)volta_cuda_abi_version() == 37 ? 0 : 1; }\n')
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-c", str(src), "-I", os.path.join(ROOT, "include"),
                    "-o", str(tmp_path / "t.o")], check=True)


def test_stubbed_entry_points_are_named(built):
    """Out-of-scope reference entry points exist and fail with a message."""
    text = open(os.path.join(ROOT, "volta_zk_b200", "csrc", "unsupported.cu")).read()
    names = set(re.findall(r'extern "C" int (volta_cuda_\w+)\(', text))
    assert len(names) == 17
    assert all(n.startswith(("volta_cuda_x4", "volta_cuda_private_argmax")) for n in names)
