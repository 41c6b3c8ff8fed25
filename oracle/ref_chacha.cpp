// Reference-side cross-check (test infrastructure only): exposes the
// reference's own host-compilable FpStream expansion,
// cuda/volta_chacha8_fp.cuh (plain C++ when __CUDACC__ is undefined, lines
// 14-20), through a C function so tests can diff the oracle against it.
// Built by oracle/Makefile into oracle/_ref/ from the header where it lies.
#include <cstddef>
#include <cstdint>

#include "volta_chacha8_fp.cuh"

extern "C" void ref_chacha_fp_rows(const uint8_t* seed, uint64_t base, size_t rows, size_t count,
                                   uint64_t* out) {
    const volta::chacha8_fp::Key key = volta::chacha8_fp::key_from_seed(seed);
    for (size_t r = 0; r < rows; ++r) {
        volta::chacha8_fp::Stream s(key, base + r);
        for (size_t j = 0; j < count; ++j) out[r * count + j] = s.next_fp();
    }
}
