// gdn_prefill.cu — placeholder until the chunked prefill lands.
#include "common.cuh"

extern "C" size_t gdn_prefill_workspace_size(const gdn_prefill_args_t*) { return 0; }
extern "C" int gdn_prefill_launch(const gdn_prefill_args_t*, gdn_stream_t) { return GDN_ERR_SHAPE; }
