// Shared layout of the fused data-parallel step (kernels + host wrappers).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "optim.cuh"

namespace mmltk {

constexpr int kDdpMaxWorld = 16;
constexpr int kSmallMax = 16;  // floats per rank in the small all-reduce
constexpr int kDdpMaxBuckets = 31;  // gradient buckets per step (barrier marks are epoch * 32 + bucket + 1)

// Flag words (uint32) inside each rank's peer-visible flag buffer.
constexpr int kFlagReady = 0;                       // [world] gradient bucket ready (epoch * 32 + bucket + 1)
constexpr int kFlagDone = kFlagReady + kDdpMaxWorld;  // [world] parameters delivered (epoch)
constexpr int kFlagSmall = kFlagDone + kDdpMaxWorld;  // [world] small all-reduce (epoch)
constexpr int kFlagNorm = 64;                        // [world] u64 (epoch << 32 | sumsq bits), 8-byte aligned
constexpr int kFlagGather = kFlagNorm + 2 * kDdpMaxWorld;   // [world] byte all-gather: payload staged (epoch)
constexpr int kFlagGatherDone = kFlagGather + kDdpMaxWorld;  // [world] byte all-gather: peers' payloads read
constexpr int kFlagWords = kFlagGatherDone + kDdpMaxWorld;

// Error codes written into DdpState::status.
constexpr int kErrTimeoutReady = 1;
constexpr int kErrTimeoutNorm = 2;
constexpr int kErrTimeoutDone = 3;
constexpr int kErrTimeoutSmall = 4;
constexpr int kErrTimeoutGather = 5;

// Pointers into every rank's peer-visible buffers (index = rank).
struct DdpPeers {
    const __nv_bfloat16* grad[kDdpMaxWorld];
    __nv_bfloat16* param[kDdpMaxWorld];
    uint32_t* flags[kDdpMaxWorld];
    float* small[kDdpMaxWorld];
    int world;
    int rank;
};

// This rank's local control words.
struct DdpState {
    uint32_t* flags_local;       // my flag buffer (peers write into it)
    float* small_local;          // my small all-reduce slots [world * kSmallMax]
    uint32_t* epoch;             // step epoch (device), starts at 1
    uint32_t* small_epoch;       // small all-reduce epoch (device), starts at 1
    uint32_t* gather_epoch;      // byte all-gather epoch (device), starts at 1
    unsigned int* ticket;        // zeroed grid ticket
    int* status;                 // 0 = ok, else kErrTimeout*
    long long spin_limit;        // polls before a wait gives up
};

// CTAs of one bucket's reduce-scatter: few when it overlaps the backward pass on a side stream, two
// waves when it runs alone after it.
int ddp_rs_blocks(bool overlapped);
cudaError_t launch_ddp_rs(const DdpPeers& peers, const DdpState& st, int64_t g_off, int64_t len, float* gshard_at,
                          float* partials_b, int bucket, int blocks, cudaStream_t s);
cudaError_t launch_ddp_publish(const DdpPeers& peers, const DdpState& st, const float* partials, int n,
                               cudaStream_t s);
// After the bucket reduce-scatters: every rank's reduced slices (bf16) into every rank's gradient
// buffer, so each holds the summed gradient (an all-reduce); then the "delivered" barrier and the
// epoch advance, as after the optimizer update.
cudaError_t launch_ddp_grad_allgather(const DdpPeers& peers, const DdpState& st, const int64_t* g_off,
                                      const int64_t* len, const int64_t* l_off, int n, const float* gshard,
                                      cudaStream_t s);
// chunks: (shard-local offset, length, group); gdelta[c]: flat offset - shard-local offset of chunk c
cudaError_t launch_ddp_update(const DdpPeers& peers, const DdpState& st, const ChunkDesc* chunks, const int64_t* gdelta,
                              int nchunks, const float* gshard, float* master, float* m, float* v, float* ema,
                              const GroupHyper* groups, const StepScalars* sc, int* flags, cudaStream_t s);
cudaError_t launch_small_allreduce(const DdpPeers& peers, const DdpState& st, float* data, int n, cudaStream_t s);
// Byte all-gather between steps: every rank has staged its payload at the start of its own gradient
// buffer; peer j's len16[j] 16-byte words land at out + off16[j].  Three launches: staged barrier,
// peer-read copy, read-done barrier (after which every gradient buffer may be written again).
cudaError_t launch_gather_bytes(const DdpPeers& peers, const DdpState& st, void* out, const int64_t* off16,
                                const int64_t* len16, cudaStream_t s);

}  // namespace mmltk
