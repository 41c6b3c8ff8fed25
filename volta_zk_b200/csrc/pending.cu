// Entry points whose B200 kernels are not in this build yet: each fails loudly.
#include "runtime.cuh"

using namespace vzb;

namespace {
int pending(void* raw, const char* what) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    const std::string m = std::string(what) + " is not implemented in this build yet";
    return reject(c, m.c_str());
}
}  // namespace

extern "C" int volta_cuda_attention_proof_wires_device(void* ctx, const vz_attention_wires_args* args) {
    return pending(ctx, "volta_cuda_attention_proof_wires_device");
}

