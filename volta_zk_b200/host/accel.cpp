// Loader, Backend and FpStream of the host mirror (see accel.hpp).
#include "accel.hpp"

#include <dlfcn.h>

#include <cstdlib>
#include <cstring>
#include <memory>

#include "api.hpp"

namespace vzh {

constexpr uint32_t kAbiVersion = 37;  // rust/volta-accel/src/lib.rs:21


// ---------------------------------------------------------------------------
// FpStream
// ---------------------------------------------------------------------------

static inline uint32_t rotl(uint32_t x, int n) { return (x << n) | (x >> (32 - n)); }

FpStream::FpStream(const uint8_t seed[32], uint64_t domain) : stream_(domain) {
    for (int i = 0; i < 8; ++i)
        key_[i] = static_cast<uint32_t>(seed[4 * i]) | (static_cast<uint32_t>(seed[4 * i + 1]) << 8) |
                  (static_cast<uint32_t>(seed[4 * i + 2]) << 16) |
                  (static_cast<uint32_t>(seed[4 * i + 3]) << 24);
}

uint64_t FpStream::next_u64() {
    if (idx_ == 8) {
        uint32_t x[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                          key_[0], key_[1], key_[2], key_[3], key_[4], key_[5], key_[6], key_[7],
                          static_cast<uint32_t>(counter_), static_cast<uint32_t>(counter_ >> 32),
                          static_cast<uint32_t>(stream_), static_cast<uint32_t>(stream_ >> 32)};
        uint32_t s[16];
        std::memcpy(s, x, sizeof s);
        auto qr = [&](int a, int b, int c, int d) {
            s[a] += s[b]; s[d] = rotl(s[d] ^ s[a], 16);
            s[c] += s[d]; s[b] = rotl(s[b] ^ s[c], 12);
            s[a] += s[b]; s[d] = rotl(s[d] ^ s[a], 8);
            s[c] += s[d]; s[b] = rotl(s[b] ^ s[c], 7);
        };
        for (int r = 0; r < 4; ++r) {
            qr(0, 4, 8, 12); qr(1, 5, 9, 13); qr(2, 6, 10, 14); qr(3, 7, 11, 15);
            qr(0, 5, 10, 15); qr(1, 6, 11, 12); qr(2, 7, 8, 13); qr(3, 4, 9, 14);
        }
        for (int i = 0; i < 16; ++i) words_[i] = s[i] + x[i];
        ++counter_;
        idx_ = 0;
    }
    const uint64_t v = static_cast<uint64_t>(words_[2 * idx_]) |
                       (static_cast<uint64_t>(words_[2 * idx_ + 1]) << 32);
    ++idx_;
    return v;
}

uint64_t FpStream::next_fp() {
    for (;;) {
        const uint64_t v = next_u64();
        if (v < vzb::kP) return v;
    }
}

// ---------------------------------------------------------------------------
// Backend
// ---------------------------------------------------------------------------

static std::string default_library() {
    if (const char* env = std::getenv("VOLTA_CUDA_LIBRARY")) return env;
    Dl_info info{};
    if (dladdr(reinterpret_cast<void*>(&default_library), &info) && info.dli_fname) {
        std::string self = info.dli_fname;
        const size_t slash = self.rfind('/');
        if (slash != std::string::npos) return self.substr(0, slash + 1) + "libvolta_cuda_backend.so";
    }
    return "libvolta_cuda_backend.so";
}

Backend::Backend(const std::string& library, TimingPolicy policy) {
    const std::string path = library.empty() ? default_library() : library;
    handle_ = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
    if (!handle_) {
        const char* e = dlerror();
        throw AccelError(std::string("LibraryLoad: ") + (e ? e : path));
    }
    std::unique_ptr<Api> api(new Api());
#define VZH_LOAD(name)                                                               \
    api->name = reinterpret_cast<decltype(api->name)>(dlsym(handle_, #name));        \
    if (!api->name) {                                                                \
        dlclose(handle_);                                                            \
        handle_ = nullptr;                                                           \
        throw AccelError("MissingSymbol: " #name);                                   \
    }
    VZH_ABI_SYMBOLS(VZH_LOAD)
#undef VZH_LOAD
    const uint32_t version = api->volta_cuda_abi_version();
    if (version != kAbiVersion) {
        dlclose(handle_);
        handle_ = nullptr;
        throw AccelError("AbiMismatch: expected " + std::to_string(kAbiVersion) + ", found " +
                         std::to_string(version));
    }
    api_ = api.release();
    ext_loaded_ = new ExtApi();
    ext_loaded_->triple_fold_round = reinterpret_cast<decltype(ext_loaded_->triple_fold_round)>(
        dlsym(handle_, "volta_b200_triple_fold_round_device"));
    ext_loaded_->logup_fold_round = reinterpret_cast<decltype(ext_loaded_->logup_fold_round)>(
        dlsym(handle_, "volta_b200_logup_fold_round_device"));
    ext_loaded_->triple_fold_round_into = reinterpret_cast<decltype(ext_loaded_->triple_fold_round_into)>(
        dlsym(handle_, "volta_b200_triple_fold_round_into_device"));
    ext_loaded_->logup_fold_round_into = reinterpret_cast<decltype(ext_loaded_->logup_fold_round_into)>(
        dlsym(handle_, "volta_b200_logup_fold_round_into_device"));
    ext_loaded_->logup_layers = reinterpret_cast<decltype(ext_loaded_->logup_layers)>(
        dlsym(handle_, "volta_b200_logup_layers_device"));
    ext_loaded_->triple_tail = reinterpret_cast<decltype(ext_loaded_->triple_tail)>(
        dlsym(handle_, "volta_b200_triple_tail_device"));
    ext_loaded_->logup_round_il = reinterpret_cast<decltype(ext_loaded_->logup_round_il)>(
        dlsym(handle_, "volta_b200_logup_round_il_into_device"));
    ext_loaded_->logup_fold_round_il = reinterpret_cast<decltype(ext_loaded_->logup_fold_round_il)>(
        dlsym(handle_, "volta_b200_logup_fold_round_il_into_device"));
    ext_loaded_->logup_round_batch = reinterpret_cast<decltype(ext_loaded_->logup_round_batch)>(
        dlsym(handle_, "volta_b200_logup_round_batch_device"));
    ext_loaded_->logup_suffix_eq_batch = reinterpret_cast<decltype(ext_loaded_->logup_suffix_eq_batch)>(
        dlsym(handle_, "volta_b200_logup_suffix_eq_batch_device"));
    ext_loaded_->triple_round_fp = reinterpret_cast<decltype(ext_loaded_->triple_round_fp)>(
        dlsym(handle_, "volta_b200_triple_round_fp_into_device"));
    ext_loaded_->triple_fold_round_fp = reinterpret_cast<decltype(ext_loaded_->triple_fold_round_fp)>(
        dlsym(handle_, "volta_b200_triple_fold_round_fp_into_device"));
    ext_loaded_->wait_uploads =
        reinterpret_cast<decltype(ext_loaded_->wait_uploads)>(dlsym(handle_, "volta_b200_wait_uploads"));
    ext_loaded_->upload_async =
        reinterpret_cast<decltype(ext_loaded_->upload_async)>(dlsym(handle_, "volta_b200_upload_async"));
    ext_loaded_->download_async =
        reinterpret_cast<decltype(ext_loaded_->download_async)>(dlsym(handle_, "volta_b200_download_async"));
    ext_loaded_->wait_downloads =
        reinterpret_cast<decltype(ext_loaded_->wait_downloads)>(dlsym(handle_, "volta_b200_wait_downloads"));
    ext_loaded_->logup_tree_column = reinterpret_cast<decltype(ext_loaded_->logup_tree_column)>(
        dlsym(handle_, "volta_b200_logup_tree_column_device"));
    ext_loaded_->triple_local = reinterpret_cast<decltype(ext_loaded_->triple_local)>(
        dlsym(handle_, "volta_b200_triple_local_device"));
    ext_loaded_->triple_flush = reinterpret_cast<decltype(ext_loaded_->triple_flush)>(
        dlsym(handle_, "volta_b200_triple_flush_device"));
    ext_loaded_->softmax_lookup_columns = reinterpret_cast<decltype(ext_loaded_->softmax_lookup_columns)>(
        dlsym(handle_, "volta_b200_softmax_lookup_columns_device"));
    ext_loaded_->av_factors =
        reinterpret_cast<decltype(ext_loaded_->av_factors)>(dlsym(handle_, "volta_b200_av_factors_device"));
    ext_loaded_->softmax_lookup_columns_band = reinterpret_cast<decltype(ext_loaded_->softmax_lookup_columns_band)>(
        dlsym(handle_, "volta_b200_softmax_lookup_columns_band_device"));
    ext_loaded_->av_factors_band = reinterpret_cast<decltype(ext_loaded_->av_factors_band)>(
        dlsym(handle_, "volta_b200_av_factors_band_device"));
    ext_loaded_->product_fold_round = reinterpret_cast<decltype(ext_loaded_->product_fold_round)>(
        dlsym(handle_, "volta_b200_product_fold_round_into_device"));
    ext_loaded_->product_tail =
        reinterpret_cast<decltype(ext_loaded_->product_tail)>(dlsym(handle_, "volta_b200_product_tail_device"));
    ext_loaded_->pack_pair_column = reinterpret_cast<decltype(ext_loaded_->pack_pair_column)>(
        dlsym(handle_, "volta_b200_pack_pair_column_device"));
    ext_loaded_->argmax_i64 =
        reinterpret_cast<decltype(ext_loaded_->argmax_i64)>(dlsym(handle_, "volta_b200_argmax_i64_device"));
    ext_loaded_->copy_segments =
        reinterpret_cast<decltype(ext_loaded_->copy_segments)>(dlsym(handle_, "volta_b200_copy_segments_device"));
    ext_loaded_->upload_batch =
        reinterpret_cast<decltype(ext_loaded_->upload_batch)>(dlsym(handle_, "volta_b200_upload_batch"));
    ext_loaded_->hash_fp_column_cvs = reinterpret_cast<decltype(ext_loaded_->hash_fp_column_cvs)>(
        dlsym(handle_, "volta_b200_hash_fp_column_cvs_device"));
    ext_ = ext_loaded_;
    void* ctx = nullptr;
    if (api_->volta_cuda_create(&ctx) != 0) {
        std::string msg = ctx ? api_->volta_cuda_last_error(ctx) : "volta_cuda_create failed";
        if (ctx) api_->volta_cuda_destroy(ctx);
        delete api_;
        api_ = nullptr;
        delete ext_loaded_;
        ext_ = ext_loaded_ = nullptr;
        dlclose(handle_);
        handle_ = nullptr;
        throw AccelError("Cuda: " + msg);
    }
    ctx_ = ctx;
    check(api_->volta_cuda_set_resident_timing_policy(ctx_, static_cast<int>(policy)),
          "set_resident_timing_policy");
}

Backend::~Backend() {
    if (api_ && ctx_) api_->volta_cuda_destroy(ctx_);
    delete api_;
    if (ext_ != ext_loaded_) delete ext_;
    delete ext_loaded_;
    if (handle_) dlclose(handle_);
}

void Backend::set_fused(bool on) {
    static const ExtApi none{};
    if (ext_ != ext_loaded_) delete ext_;
    ext_ = on ? ext_loaded_ : new ExtApi(none);
}

void Backend::raise(const char* what) const {
    throw AccelError(std::string("Cuda: ") + what + ": " + api_->volta_cuda_last_error(ctx_));
}

uint64_t Backend::alloc(size_t bytes) {
    uint64_t id = 0;
    check(api_->volta_cuda_resident_alloc(ctx_, bytes ? bytes : 16, &id), "resident_alloc");
    return id;
}

void Backend::free(uint64_t id) { check(api_->volta_cuda_resident_free(ctx_, id), "resident_free"); }

void Backend::upload(uint64_t id, size_t off, const void* src, size_t bytes) {
    check(api_->volta_cuda_resident_upload(ctx_, id, off, src, bytes), "resident_upload");
}

void Backend::download(uint64_t id, size_t off, void* dst, size_t bytes) {
    check(api_->volta_cuda_resident_download(ctx_, id, off, dst, bytes), "resident_download");
}

std::vector<Fp2> Backend::download_fp2_segments(const std::vector<std::pair<uint64_t, size_t>>& elems) {
    const size_t total = elems.size();
    const uint64_t mailbox = alloc(total * sizeof(Fp2));
    size_t before = 0, after = 0;
    int flushed = 0;
    check(api_->volta_cuda_ensure_timing_capacity(ctx_, 2, &before, &after, &flushed),
          "ensure_timing_capacity");
    check(api_->volta_cuda_begin_coarse_timing(ctx_, kMailbox), "begin_coarse_timing");
    for (size_t i = 0; i < total; ++i) {
        const int rc = api_->volta_cuda_resident_mailbox_copy_rows(
            ctx_, elems[i].first, elems[i].second * sizeof(Fp2), sizeof(Fp2), mailbox, i * sizeof(Fp2),
            sizeof(Fp2), 1, sizeof(Fp2));
        if (rc) {
            api_->volta_cuda_abort_coarse_timing(ctx_);
            raise("resident_mailbox_copy_rows");
        }
    }
    check(api_->volta_cuda_end_coarse_timing(ctx_), "end_coarse_timing");
    std::vector<Fp2> out(total);
    download(mailbox, 0, out.data(), total * sizeof(Fp2));
    free(mailbox);
    return out;
}

vz_raw_stats Backend::stats() {
    vz_raw_stats s{};
    check(api_->volta_cuda_get_stats(ctx_, &s), "get_stats");
    return s;
}

void Backend::reset_stats() { check(api_->volta_cuda_reset_stats(ctx_), "reset_stats"); }

}  // namespace vzh
