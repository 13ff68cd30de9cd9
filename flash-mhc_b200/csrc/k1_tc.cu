// K1 forward on the tensor cores: placeholder until the tcgen05 kernel lands.
#include "k1_tc.h"

namespace fmhc {

bool k1_tc_fwd_supported(const void *, const void *, const void *, const float *, int64_t,
                         int64_t, int64_t) {
  return false;
}
int launch_k1_tc_fwd(const void *, const void *, void *, float *, int64_t, int, cudaStream_t) {
  return 2;
}
const char *k1_tc_error() { return "tensor-core K1 not built"; }

}  // namespace fmhc
