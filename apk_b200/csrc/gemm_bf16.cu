// bf16 tcgen05 persistent GEMM -- placeholder until the tensor-core kernel
// lands; every entry reports "unsupported" so the runtime fails loudly.
#include <string>
#include "../../include/apk.h"
#include "proto.h"

namespace apk {
namespace bf16 {
cudaError_t prepare(int, int, bool, int* max_ctas_per_sm) {
  *max_ctas_per_sm = 0;
  return cudaErrorNotSupported;
}
cudaError_t launch(const void*, int, int, int, bool, cudaStream_t) { return cudaErrorNotSupported; }
int smem_bytes() { return 0; }
int threads() { return 0; }
size_t params_size() { return 0; }
apk_status build_params(void*, const void*, const void*, void*, int, int, int, const void*, const void*,
                        float*, int, int, int, int, size_t, const EventProto&, const QueueProto&, long long,
                        int, std::string* err) {
  *err = "bf16 path not built";
  return APK_EUNSUPPORTED;
}
}  // namespace bf16
}  // namespace apk
