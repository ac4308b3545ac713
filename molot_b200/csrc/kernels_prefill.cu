// Prefill attention kernels for every storage type.
#include "dispatch.cuh"
#include "molot_b200.h"
#include "prefill.cuh"
#include "prefill_tc.cuh"

namespace molot {
namespace {
template <int D, class KT>
KernelRef ref() {
  return {reinterpret_cast<const void*>(&gqa_prefill_kernel<D, KT>), PrefillTile<D, KT>::kTotal};
}

template <class KT>
bool pick(int D, KernelRef* k) {
  switch (D) {
    case 64: *k = ref<64, KT>(); return true;
    case 128: *k = ref<128, KT>(); return true;
    case 256: *k = ref<256, KT>(); return true;
  }
  return false;
}
}  // namespace

bool pick_prefill_tc(int D, KernelRef* k) {
  switch (D) {
    case 64:
      *k = {reinterpret_cast<const void*>(&gqa_prefill_tc_kernel<64>), TcShape<64>::kTotal};
      return true;
    case 128:
      *k = {reinterpret_cast<const void*>(&gqa_prefill_tc_kernel<128>), TcShape<128>::kTotal};
      return true;
  }
  return false;
}

bool pick_prefill_kv(int D, int kvt, KernelRef* k) {
  switch (kvt) {
    case MOLOT_KV_BF16: return pick<__nv_bfloat16>(D, k);
    case MOLOT_KV_Q8: return pick<Q8Row>(D, k);
  }
  return pick<float>(D, k);
}

}  // namespace molot
