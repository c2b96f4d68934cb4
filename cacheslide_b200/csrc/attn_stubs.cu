// Entry points of the tensor-core prefill and split-key decode kernels that
// this build does not provide yet: they report CS_ERR_UNSUPPORTED so callers
// dispatch to cs_cope_attn.
#include "common.cuh"

extern "C" int cs_cope_attn_prefill(const cs_attn_params* p, void* stream) {
  (void)p;
  (void)stream;
  return CS_ERR_UNSUPPORTED;
}

extern "C" int64_t cs_cope_attn_decode_workspace(const cs_attn_params* p) {
  (void)p;
  return 0;
}

extern "C" int cs_cope_attn_decode(const cs_attn_params* p, void* workspace, void* stream) {
  (void)p;
  (void)workspace;
  (void)stream;
  return CS_ERR_UNSUPPORTED;
}
