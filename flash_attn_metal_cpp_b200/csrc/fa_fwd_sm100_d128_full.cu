// Instantiations of the tcgen05 attention kernel for head_dim 128, non-causal.
#include "fa_fwd_sm100.cuh"

namespace fa {
namespace sm100 {

cudaError_t launch_d128_full(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk,
                            const CUtensorMap& tv, bool qk_bf16, int out_dtype, cudaStream_t stream) {
  return qk_bf16 ? launch_out<128, false, true>(a, tq, tk, tv, out_dtype, stream)
                 : launch_out<128, false, false>(a, tq, tk, tv, out_dtype, stream);
}

}  // namespace sm100
}  // namespace fa
