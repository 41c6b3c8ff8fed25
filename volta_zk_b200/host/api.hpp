// Function table of the loaded C ABI (one typed pointer per symbol of
// include/volta_cuda_backend.h).
#pragma once

#include "../../include/volta_cuda_backend.h"
#include "abi_symbols.inc"

namespace vzh {

struct Api {
#define VZH_FIELD(name) decltype(&::name) name = nullptr;
    VZH_ABI_SYMBOLS(VZH_FIELD)
#undef VZH_FIELD
};

}  // namespace vzh
