// Kernel selection across translation units.  Each storage type's decode
// kernels (and the prefill kernels) are instantiated in a translation unit
// of their own (kernels_*.cu), which the build compiles side by side; the
// rest of the library reaches them through these functions.
#pragma once

namespace molot {

// A kernel's host-side handle and its dynamic shared memory.
struct KernelRef {
  const void* fn = nullptr;
  int smem = 0;
};

// gqa_decode_kernel for a head_dim / group size and a cache storage type
// (molot_kv_dtype).  split: the FP32 kernel with split K/V stage barriers
// (head_dim <= 128).  false when that combination is not built.
bool pick_decode_f32(int D, int G, bool split, KernelRef* k);
bool pick_decode_bf16(int D, int G, KernelRef* k);
bool pick_decode_q8(int D, int G, KernelRef* k);
// gqa_prefill_kernel for a head_dim and a storage type.
bool pick_prefill_kv(int D, int kvt, KernelRef* k);

}  // namespace molot
