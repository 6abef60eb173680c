// Shared declarations of the fused optimizer (single-GPU and DDP paths).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mmltk {

// One contiguous piece of one parameter (all parameters of a chunk share a group).
struct ChunkDesc {
    int64_t offset;
    int64_t length;
    int64_t group;
};

struct GroupHyper {
    float lr;
    float weight_decay;
};

// Per-step scalars refreshed by the host (one small async copy per step).
struct StepScalars {
    float lr_scale;
    float beta1;
    float beta2;
    float eps;
    float bias_corr1;   // 1 - beta1^t
    float bias_corr2;   // 1 - beta2^t
    float max_norm;     // <= 0 disables clipping
    float ema_decay;    // effective decay for this step
    float ema_enabled;  // 0 / 1
    float inv_world;    // 1 / world size (DDP gradient average)
    float pad[6];
};
constexpr int kStepScalarFloats = sizeof(StepScalars) / sizeof(float);

int optim_num_partials();
void launch_grad_sumsq(const __nv_bfloat16* grad, int64_t n, float* partials, int nparts, cudaStream_t st);
void launch_adamw_ema(const ChunkDesc* chunks, int nchunks, const __nv_bfloat16* grad, float* master, float* m,
                      float* v, float* ema, __nv_bfloat16* param, const GroupHyper* groups, const StepScalars* sc,
                      const float* partials, int nparts, int* flags, cudaStream_t st);

}  // namespace mmltk
