// decode_d80_contig.cu -- decode_splitk_kernel instantiations for head dim 80,
// contiguous layouts (per-channel, per-token).
#include "decode_dispatch.cuh"

namespace slmt {

DecodeFn decode_fn_80_contig(int nt, bool pk, int layout, int kvc) { return contig_fn_d<80>(nt, pk, layout, kvc); }

}  // namespace slmt
