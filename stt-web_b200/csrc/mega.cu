// Persistent single-stream decode step.  Not enabled yet: mega_supported() returns false, so
// every batch size runs the captured multi-kernel step of kernels.cu.
#include "mega.h"

namespace stt {

bool mega_supported(int, int, int, int) { return false; }
size_t mega_scratch_bytes(int, int, int, int, int, int) { return 256; }
cudaError_t configure_mega() { return cudaSuccess; }
cudaError_t launch_mega_steps(MegaState&, const Ctx&, const LayerDev*, int, cudaStream_t) {
    return cudaErrorNotSupported;
}

}  // namespace stt
