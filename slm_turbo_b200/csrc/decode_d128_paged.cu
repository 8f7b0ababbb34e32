// decode_d128_paged.cu -- decode_splitk_kernel instantiations for head dim 128,
// paged per-token layout (plain and fused-append).
#include "decode_dispatch.cuh"

namespace slmt {

DecodeFn decode_fn_128_paged(int nt, bool pk, int kvc, bool append, bool swz) {
  return paged_fn_d<128>(nt, pk, kvc, append, swz);
}

}  // namespace slmt
