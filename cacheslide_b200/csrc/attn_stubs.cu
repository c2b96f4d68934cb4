// Entry point of the tensor-core prefill kernel while this build does not
// provide it: it reports CS_ERR_UNSUPPORTED so callers dispatch to
// cs_cope_attn.
#include "common.cuh"

extern "C" int cs_cope_attn_prefill(const cs_attn_params* p, void* stream) {
  (void)p;
  (void)stream;
  return CS_ERR_UNSUPPORTED;
}
