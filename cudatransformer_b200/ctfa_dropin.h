// Helpers shared by the C++ drop-ins (FlashAttentionLayer.cu,
// QKVProjectionLayer.cu, OutputProjectionLayer.cu): the element-type code of
// each DType the reference instantiates (cuda_transformer.cu:839-842) and the
// conversion of a library status into std::runtime_error.
#ifndef CTFA_DROPIN_COMMON_H
#define CTFA_DROPIN_COMMON_H

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <stdexcept>
#include <string>

#include "ctfa.h"

namespace ctfa_dropin {

template <typename T>
struct DtypeCode;
template <>
struct DtypeCode<float> {
  static constexpr int value = CTFA_DTYPE_F32;
};
template <>
struct DtypeCode<__nv_bfloat16> {
  static constexpr int value = CTFA_DTYPE_BF16;
};
template <>
struct DtypeCode<__half> {
  static constexpr int value = CTFA_DTYPE_F16;
};
template <>
struct DtypeCode<double> {
  static constexpr int value = CTFA_DTYPE_F64;
};

inline void check(int status, const char* where) {
  if (status != CTFA_OK)
    throw std::runtime_error(std::string(where) + ": " + ctfa_status_string(status) + ": " +
                             ctfa_last_error_message());
}

}  // namespace ctfa_dropin

#endif  // CTFA_DROPIN_COMMON_H
