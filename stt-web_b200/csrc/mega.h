// Persistent single-stream decode step (one launch runs whole frames); see mega.cu.
#pragma once

#include "device.cuh"

namespace stt {

struct MegaState {
    void* scratch = nullptr;  // device scratch owned by the stream set
    size_t scratch_bytes = 0;
    float* xa_all = nullptr;              // [steps][D] audio sums of the call (grown by the caller)
    unsigned long long* trace = nullptr;  // device buffer for phase timestamps (diagnostics)
    int trace_frame = -1;
    int trace_cap = 0;
    unsigned long long* trace_ctas = nullptr;  // [num_sms][trace_slots] %globaltimer per CTA
    int trace_slots = 0;
    int stall_next = 0;  // the next launch runs the bounded-wait test (one launch only)
};

// Trace slots per CTA of one frame: 1 + 16 per layer + 4 (layers <= 32).
constexpr int kTraceSlots = 1 + 16 * 32 + 4;

bool mega_supported(int L, int D, int F, int HD, int V, int num_sms, int ML, int kv_f32);
size_t mega_scratch_bytes(int num_sms, int D, int F, int V, int H, int HD);
cudaError_t configure_mega();
cudaError_t mega_barrier_probe(void* scratch, int iters, int mode, float* ms_out);
cudaError_t launch_mega_steps(MegaState& ms, const Ctx& c, const LayerDev* h_layers, int steps, cudaStream_t st);

}  // namespace stt
