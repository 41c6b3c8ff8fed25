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

extern "C" int volta_cuda_fixed_embed_device(void* ctx, uint64_t tokens_id, size_t tokens_offset, uint64_t wte_id, size_t wte_offset, uint64_t wpe_id, size_t wpe_offset, uint64_t acc_id, size_t acc_offset, uint64_t out_id, size_t out_offset, uint64_t error_id, size_t error_offset, size_t rows, size_t d, size_t vocab, size_t positions, size_t pos0, int32_t shift) {
    return pending(ctx, "volta_cuda_fixed_embed_device");
}

extern "C" int volta_cuda_fixed_layer_norm_device(void* ctx, uint64_t input_id, size_t input_offset, uint64_t gain_id, size_t gain_offset, uint64_t bias_id, size_t bias_offset, uint64_t lut_id, size_t lut_offset, uint64_t mean_id, size_t mean_offset, uint64_t var_id, size_t var_offset, uint64_t rin_id, size_t rin_offset, uint64_t rout_id, size_t rout_offset, uint64_t acc_id, size_t acc_offset, uint64_t out_id, size_t out_offset, uint64_t error_id, size_t error_offset, size_t rows, size_t d, uint32_t var_shift, uint32_t norm_shift) {
    return pending(ctx, "volta_cuda_fixed_layer_norm_device");
}

extern "C" int volta_cuda_fixed_gemm_device(void* ctx, uint64_t input_id, size_t input_offset, uint64_t weights_id, size_t weights_offset, uint64_t bias_id, size_t bias_offset, uint64_t residual_id, size_t residual_offset, uint64_t acc_id, size_t acc_offset, uint64_t requant_id, size_t requant_offset, uint64_t residual_out_id, size_t residual_out_offset, uint64_t error_id, size_t error_offset, size_t m, size_t k, size_t n, uint32_t shift) {
    return pending(ctx, "volta_cuda_fixed_gemm_device");
}

extern "C" int volta_cuda_fixed_qkv_split_device(void* ctx, uint64_t input_id, size_t input_offset, uint64_t q_id, size_t q_offset, uint64_t k_id, size_t k_offset, uint64_t v_id, size_t v_offset, size_t rows, size_t d) {
    return pending(ctx, "volta_cuda_fixed_qkv_split_device");
}

extern "C" int volta_cuda_fixed_attention_scores_device(void* ctx, uint64_t q_id, size_t q_offset, uint64_t k_id, size_t k_offset, uint64_t acc_id, size_t acc_offset, uint64_t out_id, size_t out_offset, uint64_t error_id, size_t error_offset, size_t rows, size_t seq, size_t pos0, size_t heads, size_t head_dim, uint32_t shift) {
    return pending(ctx, "volta_cuda_fixed_attention_scores_device");
}

extern "C" int volta_cuda_fixed_softmax_device(void* ctx, uint64_t scores_id, size_t scores_offset, uint64_t exp_lut_id, size_t exp_lut_offset, uint64_t recip_lut_id, size_t recip_lut_offset, uint64_t row_shift_id, size_t row_shift_offset, uint64_t exp_id, size_t exp_offset, uint64_t denoms_id, size_t denoms_offset, uint64_t recips_id, size_t recips_offset, uint64_t weights_id, size_t weights_offset, uint64_t error_id, size_t error_offset, size_t rows, size_t seq, size_t pos0, size_t heads, uint32_t recip_den_shift, uint32_t recip_log2, uint32_t norm_shift, int use_row_shift) {
    return pending(ctx, "volta_cuda_fixed_softmax_device");
}

extern "C" int volta_cuda_fixed_av_device(void* ctx, uint64_t weights_id, size_t weights_offset, uint64_t values_id, size_t values_offset, uint64_t acc_id, size_t acc_offset, uint64_t out_id, size_t out_offset, uint64_t error_id, size_t error_offset, size_t rows, size_t seq, size_t pos0, size_t d, size_t heads, uint32_t shift) {
    return pending(ctx, "volta_cuda_fixed_av_device");
}

extern "C" int volta_cuda_fixed_lookup_device(void* ctx, uint64_t input_id, size_t input_offset, uint64_t lut_id, size_t lut_offset, uint64_t out_id, size_t out_offset, size_t n) {
    return pending(ctx, "volta_cuda_fixed_lookup_device");
}

extern "C" int volta_cuda_fixed_requant_i16_device(void* ctx, uint64_t input_id, size_t input_offset, uint64_t out_id, size_t out_offset, uint64_t error_id, size_t error_offset, size_t n, uint32_t shift) {
    return pending(ctx, "volta_cuda_fixed_requant_i16_device");
}

extern "C" int volta_cuda_fixed_logits_device(void* ctx, uint64_t input_id, size_t input_offset, uint64_t weights_id, size_t weights_offset, uint64_t out_id, size_t out_offset, size_t rows, size_t d, size_t vocab) {
    return pending(ctx, "volta_cuda_fixed_logits_device");
}

extern "C" int volta_cuda_attention_proof_wires_device(void* ctx, const vz_attention_wires_args* args) {
    return pending(ctx, "volta_cuda_attention_proof_wires_device");
}

