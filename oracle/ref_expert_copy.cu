// TEST INFRASTRUCTURE ONLY: a C entry point over the reference's own fused multi-bank
// expert-slot copy kernel, compiled from the reference source tree where it lies (see
// oracle/build_ref.py) into oracle/_ref/. It exists to pin pi_expert_slot_copy bit for
// bit against the reference on the GPU and to time it beside ours; nothing in the
// product links it.
//
// The reference instantiates MultiIndexCopyKernel<num_threads, blocks_per_bank> with its
// defaults 1024 / 8 (src/plastic_infer/kernel/fast_index_copy.py:208-218) behind the
// same C signature (fast_index_copy.py:190-201); this file declares that entry point
// under its own name for the same template arguments.
#include <cstdint>

#include "fast_index_copy.cuh"  // src/plastic_infer/kernel/csrc/jit/ of the reference

extern "C" void ref_fast_index_copy_multi_launch(const int64_t* dst_ptrs, const int64_t* src_ptrs,
                                                 const int64_t* feat_bytes, const void* dst_indices,
                                                 const void* src_indices, int64_t length,
                                                 const int64_t* num_indices, int num_banks,
                                                 int use_int32, cudaStream_t stream) {
  MultiIndexCopyKernel<1024, 8>::run(dst_ptrs, src_ptrs, feat_bytes, dst_indices, src_indices,
                                     static_cast<std::size_t>(length), num_indices, num_banks,
                                     use_int32 != 0, stream);
}
