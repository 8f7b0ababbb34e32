// decode_dispatch.cuh -- picks the decode_splitk_kernel instantiation for a
// call.  Included by the per-head-dim translation units (decode_d*.cu), each
// of which instantiates its share of the kernels.
#pragma once

#include "decode_kernels.cuh"

namespace slmt {

// Instantiated per head dim, n-tiles, kv heads per CTA (compile-time row
// strides, one consumer warp per kv head) and tile packing (PK: at most 4
// query heads per kv head, so two tiles share one n-tile).  The paged
// layout has a second instantiation that also appends the step's new tokens,
// and, for whole rows of 8 kv heads at head dim 64 / 128, swizzled-stage
// variants of both (paged mode 4).
template <int D, int NT, bool PK, int KVC>
DecodeFn paged_fn(bool append, bool swz) {
  if constexpr (KVC == 8 && (D == 64 || D == 128)) {
    if (swz)
      return append ? decode_splitk_kernel<D, NT, LAYOUT_PAGED, KVC, PK, true, true>
                    : decode_splitk_kernel<D, NT, LAYOUT_PAGED, KVC, PK, false, true>;
  }
  return append ? decode_splitk_kernel<D, NT, LAYOUT_PAGED, KVC, PK, true>
                : decode_splitk_kernel<D, NT, LAYOUT_PAGED, KVC, PK, false>;
}

template <int D, int NT, bool PK, int KVC>
DecodeFn contig_fn(int layout) {
  return layout == LAYOUT_PER_CHANNEL ? decode_splitk_kernel<D, NT, LAYOUT_PER_CHANNEL, KVC, PK>
                                      : decode_splitk_kernel<D, NT, LAYOUT_PER_TOKEN, KVC, PK>;
}

template <int D, int NT, bool PK>
DecodeFn paged_fn_kvc(int kvc, bool append, bool swz) {
  switch (kvc) {
    case 8: return paged_fn<D, NT, PK, 8>(append, swz);
    case 4: return paged_fn<D, NT, PK, 4>(append, false);
    case 2: return paged_fn<D, NT, PK, 2>(append, false);
    default: return paged_fn<D, NT, PK, 1>(append, false);
  }
}

template <int D, int NT, bool PK>
DecodeFn contig_fn_kvc(int layout, int kvc) {
  switch (kvc) {
    case 8: return contig_fn<D, NT, PK, 8>(layout);
    case 4: return contig_fn<D, NT, PK, 4>(layout);
    case 2: return contig_fn<D, NT, PK, 2>(layout);
    default: return contig_fn<D, NT, PK, 1>(layout);
  }
}

template <int D>
DecodeFn paged_fn_d(int nt, bool pk, int kvc, bool append, bool swz) {
  if (nt == 2) return paged_fn_kvc<D, 2, false>(kvc, append, swz);
  return pk ? paged_fn_kvc<D, 1, true>(kvc, append, swz) : paged_fn_kvc<D, 1, false>(kvc, append, swz);
}

template <int D>
DecodeFn contig_fn_d(int nt, bool pk, int layout, int kvc) {
  if (nt == 2) return contig_fn_kvc<D, 2, false>(layout, kvc);
  return pk ? contig_fn_kvc<D, 1, true>(layout, kvc) : contig_fn_kvc<D, 1, false>(layout, kvc);
}

}  // namespace slmt
