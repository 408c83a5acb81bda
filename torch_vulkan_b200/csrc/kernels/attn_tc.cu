// Tensor-core attention (tcgen05) — placeholder until the sm_100a kernels land: nothing is eligible,
// so b2_attn_fwd/bwd route every case to the SIMT kernels.
#include "common.cuh"

namespace b2 {
bool attn_tc_eligible(const b2_attn_args*) { return false; }
int attn_tc_fwd(const b2_attn_args*, cudaStream_t) { return fail(B2_ERR_ARG, "attn_tc: not available"); }
int attn_tc_bwd(const b2_attn_args*, cudaStream_t) { return fail(B2_ERR_ARG, "attn_tc: not available"); }
}  // namespace b2

extern "C" uint64_t b2_attn_bwd_workspace_bytes(const b2_attn_args*) { return 0; }
