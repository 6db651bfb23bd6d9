// fa_fwd_sm100.cu - dispatch of the tcgen05 attention kernel
// (fa_fwd_sm100.cuh) over head_dim and the causal flag.
#include "fa_fwd_sm100.cuh"

namespace fa {

cudaError_t launch_attn_sm100(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk,
                              const CUtensorMap& tv, bool qk_bf16, int out_dtype,
                              cudaStream_t stream) {
  if (a.D == 64)
    return a.causal ? sm100::launch_d64_causal(a, tq, tk, tv, qk_bf16, out_dtype, stream)
                    : sm100::launch_d64_full(a, tq, tk, tv, qk_bf16, out_dtype, stream);
  if (a.D == 128)
    return a.causal ? sm100::launch_d128_causal(a, tq, tk, tv, qk_bf16, out_dtype, stream)
                    : sm100::launch_d128_full(a, tq, tk, tv, qk_bf16, out_dtype, stream);
  return cudaErrorInvalidValue;
}

}  // namespace fa
