// Internal glue shared by the liblaya_cuda translation units.
#pragma once
#include <string>
#include "lc_common.cuh"
#include "laya_cuda.h"

namespace lc {
void set_error(const std::string& m);
void count_launch(int n);
}  // namespace lc

// Every exported entry point runs inside LC_API_BEGIN/END: exceptions become
// a nonzero return code plus the message in lc_last_error().
#define LC_API_BEGIN try {
#define LC_API_END                                   \
  }                                                  \
  catch (const std::exception& e) {                  \
    ::lc::set_error(e.what());                       \
    return 1;                                        \
  }                                                  \
  catch (...) {                                      \
    ::lc::set_error("unknown error");                \
    return 1;                                        \
  }                                                  \
  return 0;

#define LC_LAUNCHED(n)                          \
  do {                                          \
    ::lc::count_launch(n);                      \
    CUDA_OK(cudaGetLastError());                \
  } while (0)

// Frees library-wide caches (RoPE tables, tensor maps) on lc_destroy.
void lc_internal_destroy_caches();
// Converting copy from `src` into a (possibly strided) destination view of equal shape.
void lc_internal_copy_strided(const LcTensor* src, LcTensor* dst);
