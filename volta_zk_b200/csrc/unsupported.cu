// Entry points outside this build's scope.
//
// The reference seam resolves every symbol eagerly (rust/volta-accel/src/
// cuda.rs:1159-1420), so they must exist.  They belong to the reference's
// later X4b/X4c folding-PCS generation (cuda/volta_cuda_backend.cu:5577-6543)
// and the C3 private-argmax feature (4501-4610), neither of which is on the
// prover hot path this library replaces.  Each fails loudly with a message
// and touches no device state, so a caller that reaches one learns why.
#include "runtime.cuh"

using namespace vzb;

namespace {
int unsupported(void* raw, const char* what) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    const std::string m = std::string(what) + " is unsupported in the B200 build of libvolta_cuda_backend";
    return reject(c, m.c_str());
}
}  // namespace

extern "C" int volta_cuda_private_argmax_witness_device(
    void* raw, uint64_t, size_t, uint64_t, size_t, uint64_t, size_t, uint64_t, size_t, uint64_t,
    size_t, uint64_t, size_t, uint64_t, size_t, uint64_t, size_t, uint64_t, size_t, size_t, size_t,
    size_t, size_t, size_t, size_t) {
    return unsupported(raw, "private argmax witness");
}

extern "C" int volta_cuda_private_argmax_phase_factors_device(void* raw, uint64_t, size_t, uint64_t,
                                                              size_t, uint64_t, size_t, size_t,
                                                              size_t, size_t, size_t) {
    return unsupported(raw, "private argmax phase factors");
}

extern "C" int volta_cuda_private_argmax_selector_device(void* raw, uint64_t, size_t, uint64_t, size_t,
                                                         uint64_t, size_t, size_t, size_t, size_t,
                                                         Fp2) {
    return unsupported(raw, "private argmax selector");
}

extern "C" int volta_cuda_x4b_ntt_fp2(void* raw, const Fp2*, size_t, size_t, Fp2*) {
    return unsupported(raw, "X4b Fp2 NTT");
}

extern "C" int volta_cuda_x4b_context_probe(void* raw, const uint8_t*, size_t, uint8_t*) {
    return unsupported(raw, "X4b context probe");
}

extern "C" int volta_cuda_x4b_n4_inner_tile(void* raw, const Fp2*, size_t, size_t, const uint16_t*,
                                            const uint8_t*, size_t, uint64_t, uint32_t, uint8_t,
                                            uint8_t, uint8_t*) {
    return unsupported(raw, "X4b n4 inner tile");
}

extern "C" int volta_cuda_x4b_n4_outer_nodes(void* raw, const uint8_t*, size_t, uint64_t, uint32_t,
                                             uint8_t, uint8_t, uint8_t, uint8_t*) {
    return unsupported(raw, "X4b n4 outer nodes");
}

extern "C" int volta_cuda_x4c_upload_pinned(void* raw, uint64_t, size_t, uint64_t, size_t, size_t) {
    return unsupported(raw, "X4c pinned upload");
}

extern "C" int volta_cuda_x4c_direct_fold_pinned_tile(void* raw, uint64_t, size_t, uint64_t, size_t,
                                                      size_t, size_t, size_t, size_t, uint64_t,
                                                      uint64_t) {
    return unsupported(raw, "X4c pinned direct fold");
}

extern "C" int volta_cuda_x4c_direct_fold_arena(void* raw, uint64_t, size_t, size_t, size_t, uint64_t,
                                                uint64_t) {
    return unsupported(raw, "X4c arena direct fold");
}

extern "C" int volta_cuda_x4c_activation_add_pinned_tile(void* raw, uint64_t, size_t, uint64_t,
                                                         size_t, size_t, size_t, uint64_t,
                                                         uint64_t) {
    return unsupported(raw, "X4c activation add");
}

extern "C" int volta_cuda_x4c_build_one_slot_n4(void* raw, uint64_t, size_t, size_t, size_t,
                                                const uint8_t*, uint32_t, uint8_t, uint8_t,
                                                uint8_t*) {
    return unsupported(raw, "X4c one-slot n4 build");
}

extern "C" int volta_cuda_x4c_gather_fp2_samples(void* raw, uint64_t, size_t, size_t, const uint64_t*,
                                                 size_t, Fp2*) {
    return unsupported(raw, "X4c Fp2 sample gather");
}

extern "C" int volta_cuda_x4c_batch_gather_bytes(void* raw, uint64_t, uint64_t, size_t, size_t,
                                                 size_t, size_t, size_t) {
    return unsupported(raw, "X4c batch byte gather");
}

extern "C" int volta_cuda_x4c_batch_gather_canonical_operations(void* raw, uint64_t, uint64_t,
                                                                size_t, size_t, size_t, size_t,
                                                                size_t) {
    return unsupported(raw, "X4c canonical operation gather");
}

extern "C" int volta_cuda_x4c_arena_reset(void* raw, uint64_t, size_t, size_t, int) {
    return unsupported(raw, "X4c arena reset");
}

extern "C" int volta_cuda_x4c_session_reusable_boundary(void* raw) {
    return unsupported(raw, "X4c session boundary");
}
