// BF16-cache decode kernels.
#include "decode.cuh"
#include "dispatch.cuh"

namespace molot {
namespace {
template <int D, int GS, int HS, class KT, bool SPLIT>
KernelRef ref() {
  return {reinterpret_cast<const void*>(&gqa_decode_kernel<D, GS, HS, KT, SPLIT>),
          DecodeSmem<D, GS, KT>::kTotal};
}

// Group splits: GS heads per warp, HS head sets of warps (G = GS * HS).
template <class KT, bool SPLIT>
bool pick(int D, int G, KernelRef* k) {
  switch (D) {
    case 64:
      switch (G) {
        case 1: *k = ref<64, 1, 1, KT, SPLIT>(); return true;
        case 2: *k = ref<64, 2, 1, KT, SPLIT>(); return true;
        case 4: *k = ref<64, 4, 1, KT, SPLIT>(); return true;
        case 8: *k = ref<64, 8, 1, KT, SPLIT>(); return true;
        case 16: *k = ref<64, 8, 2, KT, SPLIT>(); return true;
        case 32: *k = ref<64, 8, 4, KT, SPLIT>(); return true;
      }
      return false;
    case 128:
      switch (G) {
        case 1: *k = ref<128, 1, 1, KT, SPLIT>(); return true;
        case 2: *k = ref<128, 2, 1, KT, SPLIT>(); return true;
        case 4: *k = ref<128, 4, 1, KT, SPLIT>(); return true;
        case 8: *k = ref<128, 4, 2, KT, SPLIT>(); return true;
        case 16: *k = ref<128, 4, 4, KT, SPLIT>(); return true;
        case 32: *k = ref<128, 4, 8, KT, SPLIT>(); return true;
      }
      return false;
    case 256:
      if (SPLIT) return false;  // split stages measured slower at head_dim 256
      switch (G) {
        case 1: *k = ref<256, 1, 1, KT, false>(); return true;
        case 2: *k = ref<256, 2, 1, KT, false>(); return true;
        case 4: *k = ref<256, 2, 2, KT, false>(); return true;
        case 8: *k = ref<256, 2, 4, KT, false>(); return true;
        case 16: *k = ref<256, 2, 8, KT, false>(); return true;
      }
      return false;
  }
  return false;
}
}  // namespace

bool pick_decode_bf16(int D, int G, KernelRef* k) { return pick<__nv_bfloat16, false>(D, G, k); }

}  // namespace molot
