// Library identification and the entry points whose kernels live elsewhere.
#define CS_STR2(x) #x
#define CS_STRINGIFY(x) CS_STR2(x)
#include "common.cuh"

extern "C" const char* cs_build_info(void) {
  return "libcacheslide_sm100: sm_100a; cuda " CS_STRINGIFY(__CUDACC_VER_MAJOR__) "." CS_STRINGIFY(
      __CUDACC_VER_MINOR__);
}

extern "C" int32_t cs_abi_version(void) { return 3; }
