// Function table of the loaded C ABI (one typed pointer per symbol of
// include/volta_cuda_backend.h).
#pragma once

#include "../../include/volta_b200_ext.h"
#include "../../include/volta_cuda_backend.h"
#include "abi_symbols.inc"

namespace vzh {

struct Api {
#define VZH_FIELD(name) decltype(&::name) name = nullptr;
    VZH_ABI_SYMBOLS(VZH_FIELD)
#undef VZH_FIELD
};

// Optional extension entry points (include/volta_b200_ext.h); null when the
// loaded library is a backend without them, in which case the drivers use the
// reference's call sequence only.
struct ExtApi {
    decltype(&::volta_b200_triple_fold_round_device) triple_fold_round = nullptr;
    decltype(&::volta_b200_logup_fold_round_device) logup_fold_round = nullptr;
    decltype(&::volta_b200_triple_fold_round_into_device) triple_fold_round_into = nullptr;
    decltype(&::volta_b200_logup_fold_round_into_device) logup_fold_round_into = nullptr;
    decltype(&::volta_b200_logup_layers_device) logup_layers = nullptr;
    decltype(&::volta_b200_triple_tail_device) triple_tail = nullptr;
    decltype(&::volta_b200_logup_round_il_into_device) logup_round_il = nullptr;
    decltype(&::volta_b200_logup_fold_round_il_into_device) logup_fold_round_il = nullptr;
    decltype(&::volta_b200_logup_round_batch_device) logup_round_batch = nullptr;
    decltype(&::volta_b200_logup_suffix_eq_batch_device) logup_suffix_eq_batch = nullptr;
    decltype(&::volta_b200_triple_round_fp_into_device) triple_round_fp = nullptr;
    decltype(&::volta_b200_triple_fold_round_fp_into_device) triple_fold_round_fp = nullptr;
    decltype(&::volta_b200_wait_uploads) wait_uploads = nullptr;
    decltype(&::volta_b200_upload_async) upload_async = nullptr;
    decltype(&::volta_b200_download_async) download_async = nullptr;
    decltype(&::volta_b200_wait_downloads) wait_downloads = nullptr;
    decltype(&::volta_b200_logup_tree_column_device) logup_tree_column = nullptr;
    decltype(&::volta_b200_triple_local_device) triple_local = nullptr;
    decltype(&::volta_b200_triple_flush_device) triple_flush = nullptr;
    decltype(&::volta_b200_softmax_lookup_columns_device) softmax_lookup_columns = nullptr;
    decltype(&::volta_b200_av_factors_device) av_factors = nullptr;
    decltype(&::volta_b200_softmax_lookup_columns_band_device) softmax_lookup_columns_band = nullptr;
    decltype(&::volta_b200_av_factors_band_device) av_factors_band = nullptr;
    decltype(&::volta_b200_pack_pair_column_device) pack_pair_column = nullptr;
    decltype(&::volta_b200_product_fold_round_into_device) product_fold_round = nullptr;
    decltype(&::volta_b200_product_tail_device) product_tail = nullptr;
    decltype(&::volta_b200_argmax_i64_device) argmax_i64 = nullptr;
    decltype(&::volta_b200_copy_segments_device) copy_segments = nullptr;
    decltype(&::volta_b200_hash_fp_column_cvs_device) hash_fp_column_cvs = nullptr;
    decltype(&::volta_b200_upload_batch) upload_batch = nullptr;
};

}  // namespace vzh
