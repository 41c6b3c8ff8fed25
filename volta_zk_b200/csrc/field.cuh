// Goldilocks p = 2^64 - 2^32 + 1 and E = Fp[phi]/(phi^2 - 7) on the integer
// pipes of sm_100a.  Semantics: rust/volta-field/src/lib.rs:10-210 (every
// value that leaves a kernel is canonical in [0, p)).
//
// Reduction of a 128-bit product x = lo + 2^64 * hi uses the two published
// Goldilocks identities 2^64 = 2^32 - 1 and 2^96 = -1 (mod p):
//   x = lo - hi[63:32] + hi[31:0] * (2^32 - 1).
// Fp2 products use Karatsuba (3 base products instead of 4) and a shift-based
// multiply by the non-residue 7, so an Fp2 product costs 3 wide multiplies.
#pragma once

#include <cstdint>

#include "../../include/volta_cuda_backend.h"

namespace vzb {

constexpr uint64_t kP = 0xFFFFFFFF00000001ull;
constexpr uint64_t kEps = 0xFFFFFFFFull;  // 2^64 mod p

// The ABI's Fp2Repr; using the public header's type lets the compiler check
// every exported signature against include/volta_cuda_backend.h.
using Fp2 = ::vz_fp2;
static_assert(sizeof(Fp2) == 16 && alignof(Fp2) == 16, "Fp2Repr layout");

__host__ __device__ __forceinline__ uint64_t fadd(uint64_t a, uint64_t b) {
    uint64_t s = a + b;
    s += (s < a) ? kEps : 0;  // a + b >= 2^64: fold the carry as 2^32 - 1
    return s >= kP ? s - kP : s;
}

__host__ __device__ __forceinline__ uint64_t fsub(uint64_t a, uint64_t b) {
    const uint64_t r = a - b;
    return a < b ? r - kEps : r;  // borrow of 2^64 is -(2^32 - 1)
}

__host__ __device__ __forceinline__ uint64_t fneg(uint64_t a) { return a ? kP - a : 0; }

__host__ __device__ __forceinline__ uint64_t freduce128(uint64_t lo, uint64_t hi) {
    const uint64_t hh = hi >> 32;
    const uint64_t hl = hi & kEps;
    uint64_t t = lo - hh;
    if (lo < hh) t -= kEps;
    const uint64_t u = (hl << 32) - hl;  // hl * (2^32 - 1), never overflows
    uint64_t r = t + u;
    if (r < t) r += kEps;
    return r >= kP ? r - kP : r;
}

__host__ __device__ __forceinline__ uint64_t fmul(uint64_t a, uint64_t b) {
#ifdef __CUDA_ARCH__
    const uint64_t lo = a * b;
    const uint64_t hi = __umul64hi(a, b);
#else
    const unsigned __int128 m = static_cast<unsigned __int128>(a) * b;
    const uint64_t lo = static_cast<uint64_t>(m);
    const uint64_t hi = static_cast<uint64_t>(m >> 64);
#endif
    return freduce128(lo, hi);
}

// 7 * a for canonical a: 8a = (a << 3) + (a >> 61) * 2^64, then subtract a.
__host__ __device__ __forceinline__ uint64_t fmul7(uint64_t a) {
    const uint64_t lo = a << 3;
    const uint64_t hi = a >> 61;
    uint64_t s = lo + hi * kEps;
    if (s < lo) s += kEps;
    if (s >= kP) s -= kP;
    return fsub(s, a);
}

__host__ __device__ __forceinline__ uint64_t fpow(uint64_t b, uint64_t e) {
    uint64_t acc = 1;
    while (e) {
        if (e & 1) acc = fmul(acc, b);
        b = fmul(b, b);
        e >>= 1;
    }
    return acc;
}

// Signed embedding valid over the whole i64 range (|x| <= 2^63 < p).
__host__ __device__ __forceinline__ uint64_t ffrom_i64(int64_t x) {
    if (x >= 0) return static_cast<uint64_t>(x);
    const uint64_t mag = static_cast<uint64_t>(-(x + 1)) + 1;
    return kP - mag;
}

__host__ __device__ __forceinline__ Fp2 f2(uint64_t a, uint64_t b) { return Fp2{a, b}; }
__host__ __device__ __forceinline__ Fp2 f2zero() { return Fp2{0, 0}; }
__host__ __device__ __forceinline__ Fp2 f2one() { return Fp2{1, 0}; }

__host__ __device__ __forceinline__ Fp2 f2add(Fp2 a, Fp2 b) {
    return Fp2{fadd(a.c0, b.c0), fadd(a.c1, b.c1)};
}
__host__ __device__ __forceinline__ Fp2 f2sub(Fp2 a, Fp2 b) {
    return Fp2{fsub(a.c0, b.c0), fsub(a.c1, b.c1)};
}
__host__ __device__ __forceinline__ Fp2 f2neg(Fp2 a) { return Fp2{fneg(a.c0), fneg(a.c1)}; }

__host__ __device__ __forceinline__ Fp2 f2mul(Fp2 a, Fp2 b) {
    const uint64_t t0 = fmul(a.c0, b.c0);
    const uint64_t t1 = fmul(a.c1, b.c1);
    const uint64_t t2 = fmul(fadd(a.c0, a.c1), fadd(b.c0, b.c1));
    return Fp2{fadd(t0, fmul7(t1)), fsub(fsub(t2, t0), t1)};
}

__host__ __device__ __forceinline__ Fp2 f2mul_base(Fp2 a, uint64_t x) {
    return Fp2{fmul(a.c0, x), fmul(a.c1, x)};
}

// Line through (0, v0), (1, v1) evaluated at 2 and 3.
__host__ __device__ __forceinline__ Fp2 f2at2(Fp2 v0, Fp2 v1) {
    return f2sub(f2add(v1, v1), v0);
}
__host__ __device__ __forceinline__ Fp2 f2at3(Fp2 v0, Fp2 v1) {
    const Fp2 d = f2sub(v1, v0);
    return f2add(f2add(f2add(v0, d), d), d);
}

// fold: v0 + (v1 - v0) * r
__host__ __device__ __forceinline__ Fp2 f2fold(Fp2 v0, Fp2 v1, Fp2 r) {
    return f2add(v0, f2mul(f2sub(v1, v0), r));
}

__host__ __device__ __forceinline__ Fp2 f2inv(Fp2 a) {
    const uint64_t norm = fsub(fmul(a.c0, a.c0), fmul7(fmul(a.c1, a.c1)));
    const uint64_t ni = fpow(norm, kP - 2);
    return Fp2{fmul(a.c0, ni), fmul(fneg(a.c1), ni)};
}

#ifdef __CUDACC__
// 128-bit read-only load of one Fp2 (16-byte aligned by the ABI).
__device__ __forceinline__ Fp2 ldg2(const Fp2* p) {
    const ulonglong2 v = __ldg(reinterpret_cast<const ulonglong2*>(p));
    return Fp2{v.x, v.y};
}
// Streaming load: data read exactly once by this launch.
__device__ __forceinline__ Fp2 ldcs2(const Fp2* p) {
    const ulonglong2 v = __ldcs(reinterpret_cast<const ulonglong2*>(p));
    return Fp2{v.x, v.y};
}
__device__ __forceinline__ void st2(Fp2* p, Fp2 v) {
    *reinterpret_cast<ulonglong2*>(p) = make_ulonglong2(v.c0, v.c1);
}
__device__ __forceinline__ Fp2 shfl_down2(Fp2 v, int d) {
    return Fp2{__shfl_down_sync(0xFFFFFFFFu, v.c0, d), __shfl_down_sync(0xFFFFFFFFu, v.c1, d)};
}
#endif

}  // namespace vzb
