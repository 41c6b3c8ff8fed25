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

#ifdef __CUDACC__
// ---------------------------------------------------------------------------
// Device arithmetic on 32-bit limbs with carry chains.
//
// The 64-bit C++ forms above compile to compare/select sequences on the
// integer ALU pipe, which ncu showed saturated (85 %) while the IMAD pipe sat
// at 14 %.  These forms keep products on IMAD (mul/mad .lo/.hi with carry)
// and use the carry flag instead of compares.  Wide values are little-endian
// u32 limbs.
// ---------------------------------------------------------------------------

struct W5 {  // up to 160-bit unsigned value: sum of 128-bit products
    uint32_t w[5];
};

__device__ __forceinline__ uint32_t lo32(uint64_t x) { return static_cast<uint32_t>(x); }
__device__ __forceinline__ uint32_t hi32(uint64_t x) { return static_cast<uint32_t>(x >> 32); }
__device__ __forceinline__ uint64_t pack64(uint32_t lo, uint32_t hi) {
    return static_cast<uint64_t>(lo) | (static_cast<uint64_t>(hi) << 32);
}

// canonical a + b (a, b < p): r = a - (p - b), add p back on borrow
__device__ __forceinline__ uint64_t dadd(uint64_t a, uint64_t b) {
    uint32_t r0, r1;
    asm("{\n\t.reg .u32 n0, n1, t0, t1, m, m0;\n\t"
        "sub.cc.u32  n0, 1, %3;\n\t"
        "subc.u32    n1, 0xFFFFFFFF, %4;\n\t"
        "sub.cc.u32  t0, %2, n0;\n\t"
        "subc.cc.u32 t1, %5, n1;\n\t"
        "subc.u32    m, 0, 0;\n\t"
        "and.b32     m0, m, 1;\n\t"
        "add.cc.u32  %0, t0, m0;\n\t"
        "addc.u32    %1, t1, m;\n\t}"
        : "=r"(r0), "=r"(r1)
        : "r"(lo32(a)), "r"(lo32(b)), "r"(hi32(b)), "r"(hi32(a)));
    return pack64(r0, r1);
}

// canonical a - b: add p back on borrow
__device__ __forceinline__ uint64_t dsub(uint64_t a, uint64_t b) {
    uint32_t r0, r1;
    asm("{\n\t.reg .u32 t0, t1, m, m0;\n\t"
        "sub.cc.u32  t0, %2, %4;\n\t"
        "subc.cc.u32 t1, %3, %5;\n\t"
        "subc.u32    m, 0, 0;\n\t"
        "and.b32     m0, m, 1;\n\t"
        "add.cc.u32  %0, t0, m0;\n\t"
        "addc.u32    %1, t1, m;\n\t}"
        : "=r"(r0), "=r"(r1)
        : "r"(lo32(a)), "r"(hi32(a)), "r"(lo32(b)), "r"(hi32(b)));
    return pack64(r0, r1);
}

// a + b for canonical b and any 64-bit a: result < 2^64 but possibly >= p
// ("weak"); valid as a multiplication input.  A carry is folded as 2^32 - 1,
// which cannot overflow again because b < p.
__device__ __forceinline__ uint64_t dadd_weak(uint64_t a, uint64_t b) {
    uint32_t r0, r1;
    asm("{\n\t.reg .u32 t0, t1, c;\n\t"
        "add.cc.u32  t0, %2, %4;\n\t"
        "addc.cc.u32 t1, %3, %5;\n\t"
        "addc.u32    c, 0, 0;\n\t"
        "neg.s32     c, c;\n\t"
        "add.cc.u32  %0, t0, c;\n\t"
        "addc.u32    %1, t1, 0;\n\t}"
        : "=r"(r0), "=r"(r1)
        : "r"(lo32(a)), "r"(hi32(a)), "r"(lo32(b)), "r"(hi32(b)));
    return pack64(r0, r1);
}

// full 128-bit product a*b into limbs (w[4] = 0)
__device__ __forceinline__ W5 dmul_wide(uint64_t a, uint64_t b) {
    W5 r;
    asm("mul.lo.u32     %0, %5, %7;\n\t"
        "mul.hi.u32     %1, %5, %7;\n\t"
        "mad.lo.cc.u32  %1, %5, %8, %1;\n\t"
        "madc.hi.u32    %2, %5, %8, 0;\n\t"
        "mad.lo.cc.u32  %1, %6, %7, %1;\n\t"
        "madc.hi.cc.u32 %2, %6, %7, %2;\n\t"
        "addc.u32       %3, 0, 0;\n\t"
        "mad.lo.cc.u32  %2, %6, %8, %2;\n\t"
        "madc.hi.u32    %3, %6, %8, %3;\n\t"
        "mov.u32        %4, 0;"
        : "=&r"(r.w[0]), "=&r"(r.w[1]), "=&r"(r.w[2]), "=&r"(r.w[3]), "=&r"(r.w[4])
        : "r"(lo32(a)), "r"(hi32(a)), "r"(lo32(b)), "r"(hi32(b)));
    return r;
}

// acc += x (x a 128-bit value in limbs 0..3)
__device__ __forceinline__ void wadd(W5& acc, const W5& x) {
    asm("add.cc.u32  %0, %0, %5;\n\t"
        "addc.cc.u32 %1, %1, %6;\n\t"
        "addc.cc.u32 %2, %2, %7;\n\t"
        "addc.cc.u32 %3, %3, %8;\n\t"
        "addc.u32    %4, %4, 0;"
        : "+r"(acc.w[0]), "+r"(acc.w[1]), "+r"(acc.w[2]), "+r"(acc.w[3]), "+r"(acc.w[4])
        : "r"(x.w[0]), "r"(x.w[1]), "r"(x.w[2]), "r"(x.w[3]));
}

// acc += 7 * x (x a 128-bit value), on the IMAD pipe
__device__ __forceinline__ void wadd7(W5& acc, const W5& x) {
    asm("mad.lo.cc.u32  %0, %5, 7, %0;\n\t"
        "madc.lo.cc.u32 %1, %6, 7, %1;\n\t"
        "madc.lo.cc.u32 %2, %7, 7, %2;\n\t"
        "madc.lo.cc.u32 %3, %8, 7, %3;\n\t"
        "addc.u32       %4, %4, 0;\n\t"
        "mad.hi.cc.u32  %1, %5, 7, %1;\n\t"
        "madc.hi.cc.u32 %2, %6, 7, %2;\n\t"
        "madc.hi.cc.u32 %3, %7, 7, %3;\n\t"
        "madc.hi.u32    %4, %8, 7, %4;"
        : "+r"(acc.w[0]), "+r"(acc.w[1]), "+r"(acc.w[2]), "+r"(acc.w[3]), "+r"(acc.w[4])
        : "r"(x.w[0]), "r"(x.w[1]), "r"(x.w[2]), "r"(x.w[3]));
}

// Canonical reduction of x = sum w_i 2^(32 i) with w4 < 2^31:
// x = (w1:w0) + w2 (2^32 - 1) - (w4:w3)   (2^64 = 2^32 - 1, 2^96 = -1, 2^128 = -2^32)
__device__ __forceinline__ uint64_t wreduce(const W5& x) {
    uint32_t r0, r1;
    asm("{\n\t.reg .u32 t0, t1, m, u0, u1, c, s0, s1, f;\n\t.reg .pred pf;\n\t"
        "sub.cc.u32  t0, %2, %5;\n\t"
        "subc.cc.u32 t1, %3, %6;\n\t"
        "subc.u32    m, 0, 0;\n\t"
        "sub.cc.u32  t0, t0, m;\n\t"
        "subc.u32    t1, t1, 0;\n\t"
        "sub.cc.u32  u0, 0, %4;\n\t"
        "subc.u32    u1, %4, 0;\n\t"
        "add.cc.u32  t0, t0, u0;\n\t"
        "addc.cc.u32 t1, t1, u1;\n\t"
        "addc.u32    c, 0, 0;\n\t"
        "neg.s32     c, c;\n\t"
        "add.cc.u32  t0, t0, c;\n\t"
        "addc.u32    t1, t1, 0;\n\t"
        "add.cc.u32  s0, t0, 0xFFFFFFFF;\n\t"
        "addc.cc.u32 s1, t1, 0;\n\t"
        "addc.u32    f, 0, 0;\n\t"
        "setp.ne.u32 pf, f, 0;\n\t"
        "selp.u32    %0, s0, t0, pf;\n\t"
        "selp.u32    %1, s1, t1, pf;\n\t}"
        : "=r"(r0), "=r"(r1)
        : "r"(x.w[0]), "r"(x.w[1]), "r"(x.w[2]), "r"(x.w[3]), "r"(x.w[4]));
    return pack64(r0, r1);
}

__device__ __forceinline__ uint64_t dmul(uint64_t a, uint64_t b) { return wreduce(dmul_wide(a, b)); }

// Lazily reduced Fp2 value: c0 and c1 as sums of 128-bit products.
struct Fp2W {
    W5 c0, c1;
};

__device__ __forceinline__ void f2w_zero(Fp2W& x) {
#pragma unroll
    for (int i = 0; i < 5; ++i) x.c0.w[i] = x.c1.w[i] = 0;
}

// acc += a * b (schoolbook: c0 += a0 b0 + 7 a1 b1, c1 += a0 b1 + a1 b0); a, b weak
__device__ __forceinline__ void f2w_mac(Fp2W& acc, Fp2 a, Fp2 b) {
    wadd(acc.c0, dmul_wide(a.c0, b.c0));
    wadd7(acc.c0, dmul_wide(a.c1, b.c1));
    wadd(acc.c1, dmul_wide(a.c0, b.c1));
    wadd(acc.c1, dmul_wide(a.c1, b.c0));
}

__device__ __forceinline__ Fp2 f2w_reduce(const Fp2W& x) { return Fp2{wreduce(x.c0), wreduce(x.c1)}; }

// canonical a * b for weak (any u64) components
__device__ __forceinline__ Fp2 d2mul(Fp2 a, Fp2 b) {
    Fp2W t;
    t.c0 = dmul_wide(a.c0, b.c0);
    wadd7(t.c0, dmul_wide(a.c1, b.c1));
    t.c1 = dmul_wide(a.c0, b.c1);
    wadd(t.c1, dmul_wide(a.c1, b.c0));
    return f2w_reduce(t);
}

__device__ __forceinline__ Fp2 d2add(Fp2 a, Fp2 b) { return Fp2{dadd(a.c0, b.c0), dadd(a.c1, b.c1)}; }
__device__ __forceinline__ Fp2 d2sub(Fp2 a, Fp2 b) { return Fp2{dsub(a.c0, b.c0), dsub(a.c1, b.c1)}; }
__device__ __forceinline__ Fp2 d2add_weak(Fp2 a, Fp2 b) {
    return Fp2{dadd_weak(a.c0, b.c0), dadd_weak(a.c1, b.c1)};
}
// v0 + (v1 - v0) r, canonical
__device__ __forceinline__ Fp2 d2fold(Fp2 v0, Fp2 v1, Fp2 r) { return d2add(v0, d2mul(d2sub(v1, v0), r)); }
#endif  // __CUDACC__

__host__ __device__ __forceinline__ uint64_t fadd(uint64_t a, uint64_t b) {
#ifdef __CUDA_ARCH__
    return dadd(a, b);
#endif
    // branch-free (masks instead of branches: random field values make
    // every branch a coin flip for the host's predictor)
    uint64_t s = a + b;
    s += kEps & (0 - static_cast<uint64_t>(s < a));  // a + b >= 2^64: fold the carry as 2^32 - 1
    return s - (kP & (0 - static_cast<uint64_t>(s >= kP)));
}

__host__ __device__ __forceinline__ uint64_t fsub(uint64_t a, uint64_t b) {
#ifdef __CUDA_ARCH__
    return dsub(a, b);
#endif
    const uint64_t r = a - b;
    return r - (kEps & (0 - static_cast<uint64_t>(a < b)));  // borrow of 2^64 is -(2^32 - 1)
}

__host__ __device__ __forceinline__ uint64_t fneg(uint64_t a) { return a ? kP - a : 0; }

__host__ __device__ __forceinline__ uint64_t freduce128(uint64_t lo, uint64_t hi) {
    // x = lo + 2^64 hi = lo - hh + hl (2^32 - 1) with hi = hh 2^32 + hl
    // (2^64 = 2^32 - 1, 2^96 = -1 mod p); branch-free, as fadd
    const uint64_t hh = hi >> 32;
    const uint64_t hl = hi & kEps;
    uint64_t t = lo - hh;
    t -= kEps & (0 - static_cast<uint64_t>(lo < hh));
    const uint64_t u = (hl << 32) - hl;  // hl * (2^32 - 1), never overflows
    uint64_t r = t + u;
    r += kEps & (0 - static_cast<uint64_t>(r < t));
    return r - (kP & (0 - static_cast<uint64_t>(r >= kP)));
}

__host__ __device__ __forceinline__ uint64_t fmul(uint64_t a, uint64_t b) {
#ifdef __CUDA_ARCH__
    return dmul(a, b);
#else
    const unsigned __int128 m = static_cast<unsigned __int128>(a) * b;
    const uint64_t lo = static_cast<uint64_t>(m);
    const uint64_t hi = static_cast<uint64_t>(m >> 64);
    return freduce128(lo, hi);
#endif
}

// 7 * a for canonical a: 8a = (a << 3) + (a >> 61) * 2^64, then subtract a.
__host__ __device__ __forceinline__ uint64_t fmul7(uint64_t a) {
    const uint64_t lo = a << 3;
    const uint64_t hi = a >> 61;
    uint64_t s = lo + hi * kEps;
    s += kEps & (0 - static_cast<uint64_t>(s < lo));
    s -= kP & (0 - static_cast<uint64_t>(s >= kP));
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
#ifdef __CUDA_ARCH__
    return d2mul(a, b);
#endif
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
