// Fused data-parallel gradient step over NVSwitch peer memory.
//
// Replaces the reference's `allreduce_coalesced` of every fp32 gradient after
// backward followed by a replicated `clip_grad_norm_` + fused AdamW + EMA
// (`src/rfdetr/training/train.cpp:876-887,1389-1410,2287-2344`).
//
// Every rank owns one contiguous shard of the flat parameter space.  Two
// kernels per step, both reading and writing other GPUs' memory directly
// (CUDA IPC mappings, 16-byte P2P loads and stores; no TMA, plain loads and
// stores only):
//
//   ddp_rs_kernel      per gradient bucket (launched on a side stream as the
//                      backward pass completes the bucket): barrier "bucket
//                      ready" -> reduce-scatter: sum this rank's slice of the
//                      bucket over every rank's bf16 gradient buffer in fp32
//                      (fixed rank order) into the local fp32 shard, plus the
//                      slice's sum of squares;
//   ddp_publish_kernel after the last bucket: the shard's sum of squares to
//                      every peer;
//   ddp_update_kernel  wait for every rank's sum of squares -> global L2 norm
//                      of the averaged gradient -> clip -> AdamW on the fp32
//                      master shard -> EMA shard update -> all-gather: write
//                      the new bf16 parameters into every rank's parameter
//                      buffer -> barrier "parameters delivered".
//
// Between steps the same mappings carry a byte all-gather (evaluation match
// records): each rank stages its payload in its own gradient buffer, and every
// rank reads every peer's payload straight out of that peer's buffer.
//
// Flags carry a per-step epoch (incremented on the device at the end of the
// update kernel), so the two kernels can be replayed from a CUDA graph
// without any host involvement.  Every wait is bounded: after
// `spin_limit` polls a wait records an error code in `status` (device memory
// the host reads once per step) and the kernel returns instead of hanging.
#include "common.cuh"
#include "ddp_fused.h"
#include "optim.cuh"

namespace mmltk {

namespace {

__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// 16-byte load of another GPU's memory, coherent at system scope (never served
// from a stale cache line of an earlier step)
__device__ __forceinline__ uint4 ld_peer16(const void* p) {
    uint4 r;
    asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}

__device__ __forceinline__ void bf16x8_to_f32(uint4 raw, float* f) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __bfloat1622float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// Bounded wait until *flag >= want (epochs only grow).  Returns false on timeout.
__device__ bool wait_u32(const uint32_t* flag, uint32_t want, long long spin_limit) {
    for (long long it = 0; it < spin_limit; ++it) {
        if (static_cast<int32_t>(ld_acquire_u32(flag) - want) >= 0) return true;
        __nanosleep(it < 64 ? 32 : 256);
    }
    return false;
}

__device__ void record_error(int* status, int code) { atomicCAS(status, 0, code); }

// Grid-wide "last CTA" election with a self-resetting ticket.
__device__ bool last_cta(unsigned int* ticket) {
    __shared__ bool is_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int t = atomicAdd(ticket, 1u);
        is_last = (t == gridDim.x - 1);
        if (is_last) *ticket = 0u;
    }
    __syncthreads();
    return is_last;
}

// Reduce-scatter of one gradient bucket: this rank's slice [g_off, g_off + len) of the flat gradient,
// summed over every rank's buffer in rank order (fp32), into gshard_at; per-CTA sums of squares into
// partials_b.  Starts with the bucket's barrier: mark = epoch * 32 + bucket + 1 is published to every
// rank and awaited from every rank (marks only grow within and across steps).
// The bucket barrier: publish mark = epoch * 32 + bucket + 1 to every rank, then wait (bounded) for
// every rank's mark.  Run by every CTA of the reduce-scatter when it is alone on the GPU, or by a
// one-CTA launch ahead of it when the reduce-scatter overlaps the backward pass (only 32 threads
// spin then, instead of a whole grid holding SM slots the backward kernels need).
__device__ bool bucket_barrier(const DdpPeers& peers, const DdpState& st, int bucket, bool publish) {
    const uint32_t mark = *st.epoch * 32u + static_cast<uint32_t>(bucket) + 1u;
    const int world = peers.world, rank = peers.rank;
    if (publish && threadIdx.x < world) {
        __threadfence_system();
        st_release_u32(peers.flags[threadIdx.x] + kFlagReady + rank, mark);
    }
    __shared__ int ok;
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if (threadIdx.x < world) {
        if (!wait_u32(st.flags_local + kFlagReady + threadIdx.x, mark, st.spin_limit)) {
            record_error(st.status, kErrTimeoutReady);
            ok = 0;
        }
    }
    __syncthreads();
    return ok != 0;
}

__global__ void ddp_bucket_barrier_kernel(DdpPeers peers, DdpState st, int bucket) {
    bucket_barrier(peers, st, bucket, true);
}

__global__ void __launch_bounds__(256) ddp_rs_kernel(DdpPeers peers, DdpState st, int64_t g_off, int64_t len,
                                                     float* __restrict__ gshard_at, float* __restrict__ partials_b,
                                                     int bucket, int own_barrier) {
    const int world = peers.world;
    // ---- barrier: my gradients of this bucket are complete; wait for everybody's (here, or in the
    // one-CTA launch before this one; a failed wait there left its code in the status word)
    if (own_barrier && !bucket_barrier(peers, st, bucket, blockIdx.x == 0)) {
        if (threadIdx.x == 0) partials_b[blockIdx.x] = 0.f;
        return;
    }
    // ---- reduce: every peer's 16 bytes loaded before any is added (all loads in flight at once)
    float ss = 0.f;
    const int64_t nvec = len / 8;
    for (int64_t vi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; vi < nvec;
         vi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t e = g_off + 8 * vi;
        uint4 raw[kDdpMaxWorld];
#pragma unroll
        for (int j = 0; j < kDdpMaxWorld; ++j)
            if (j < world) raw[j] = ld_peer16(peers.grad[j] + e);
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < kDdpMaxWorld; ++j) {
            if (j < world) {
                float f[8];
                bf16x8_to_f32(raw[j], f);
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[c] += f[c];
            }
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) ss += acc[c] * acc[c];
        store8(gshard_at + 8 * vi, acc);
    }
    __shared__ float red[8];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < (blockDim.x >> 5); ++w) t += red[w];
        partials_b[blockIdx.x] = t;
    }
}

// After the last bucket: this rank's sum of squares (all buckets' partials, fixed order) published to
// every rank as (epoch << 32 | bits).
__global__ void ddp_publish_kernel(DdpPeers peers, DdpState st, const float* __restrict__ partials, int n) {
    const uint32_t epoch = *st.epoch;
    float t = 0.f;
    for (int i = threadIdx.x; i < n; i += 32) t += partials[i];
    t = warp_sum(t);
    if (threadIdx.x < peers.world) {
        const unsigned long long packed = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(t);
        __threadfence_system();
        st_release_u64(reinterpret_cast<unsigned long long*>(peers.flags[threadIdx.x] + kFlagNorm) + peers.rank,
                       packed);
    }
}

__global__ void __launch_bounds__(256) ddp_update_kernel(DdpPeers peers, DdpState st,
                                                         const ChunkDesc* __restrict__ chunks,
                                                         const int64_t* __restrict__ gdelta, int nchunks,
                                                         const float* __restrict__ gshard,
                                                         float* __restrict__ master, float* __restrict__ m,
                                                         float* __restrict__ v, float* __restrict__ ema,
                                                         const GroupHyper* __restrict__ groups,
                                                         const StepScalars* __restrict__ sc, int* __restrict__ flags) {
    const uint32_t epoch = *st.epoch;
    const int world = peers.world, rank = peers.rank;
    __shared__ float s_sumsq;
    __shared__ int ok;
    if (threadIdx.x == 0) {
        ok = 1;
        s_sumsq = 0.f;
    }
    __syncthreads();
    // ---- every rank's shard sum of squares (fixed order -> same norm on every rank)
    if (threadIdx.x == 0) {
        float tot = 0.f;
        for (int j = 0; j < world; ++j) {
            const unsigned long long* slot =
                reinterpret_cast<const unsigned long long*>(st.flags_local + kFlagNorm) + j;
            unsigned long long val = 0;
            bool got = false;
            for (long long it = 0; it < st.spin_limit; ++it) {
                val = ld_acquire_u64(slot);
                if (static_cast<uint32_t>(val >> 32) == epoch) {
                    got = true;
                    break;
                }
                __nanosleep(it < 64 ? 32 : 256);
            }
            if (!got) {
                record_error(st.status, kErrTimeoutNorm);
                ok = 0;
                break;
            }
            tot += __uint_as_float(static_cast<uint32_t>(val & 0xffffffffu));
        }
        s_sumsq = tot;
    }
    __syncthreads();
    if (!ok) return;
    const float inv_world = sc->inv_world > 0.f ? sc->inv_world : 1.f;
    const float norm = sqrtf(s_sumsq) * inv_world;
    const bool finite = isfinite(norm);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (!finite) flags[0] = 1;
        reinterpret_cast<float*>(flags)[1] = norm;
    }
    float clip = 1.f;
    if (sc->max_norm > 0.f && finite) clip = fminf(1.f, sc->max_norm / (norm + 1e-6f));
    const float gs = clip * inv_world;
    const float b1 = sc->beta1, b2 = sc->beta2, eps = sc->eps;
    const float inv_bc1 = 1.f / sc->bias_corr1, inv_sqrt_bc2 = rsqrtf(sc->bias_corr2);
    const float ema_d = sc->ema_decay;
    const bool do_ema = ema != nullptr && sc->ema_enabled != 0.f;
    // ---- sharded AdamW + EMA, then all-gather of the bf16 parameters
    for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const ChunkDesc cd = chunks[c];  // offsets are shard-local; + gdelta[c] = flat offset
        const int64_t to_flat = gdelta[c];
        const GroupHyper gh = groups[cd.group];
        const float lr = gh.lr * sc->lr_scale;
        const float decay = 1.f - lr * gh.weight_decay;
        // 8 elements per thread: two float4 of every fp32 operand and one 16-byte store of the bf16
        // parameters per peer (chunks start at multiples of 8; a chunk's last group may run into the
        // parameter's zero padding, whose update keeps it zero)
        for (int64_t i = cd.offset + 8 * threadIdx.x; i < cd.offset + cd.length; i += 8 * blockDim.x) {
            float4 p[2] = {*reinterpret_cast<float4*>(master + i), *reinterpret_cast<float4*>(master + i + 4)};
            if (finite) {
                // all operands loaded before use: one memory round trip per iteration
                float4 g4[2], mm[2], vv[2], e[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    g4[h] = *reinterpret_cast<const float4*>(gshard + i + 4 * h);
                    mm[h] = *reinterpret_cast<float4*>(m + i + 4 * h);
                    vv[h] = *reinterpret_cast<float4*>(v + i + 4 * h);
                    e[h] = do_ema ? *reinterpret_cast<const float4*>(ema + i + 4 * h) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float gv[4] = {g4[h].x * gs, g4[h].y * gs, g4[h].z * gs, g4[h].w * gs};
                    float* pp = &p[h].x;
                    float* mp = &mm[h].x;
                    float* vp = &vv[h].x;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        mp[k] = b1 * mp[k] + (1.f - b1) * gv[k];
                        vp[k] = b2 * vp[k] + (1.f - b2) * gv[k] * gv[k];
                        const float denom = sqrtf(vp[k]) * inv_sqrt_bc2 + eps;
                        pp[k] = pp[k] * decay - lr * inv_bc1 * mp[k] / denom;
                    }
                    *reinterpret_cast<float4*>(master + i + 4 * h) = p[h];
                    *reinterpret_cast<float4*>(m + i + 4 * h) = mm[h];
                    *reinterpret_cast<float4*>(v + i + 4 * h) = vv[h];
                    if (do_ema) {
                        e[h].x = ema_d * e[h].x + (1.f - ema_d) * p[h].x;
                        e[h].y = ema_d * e[h].y + (1.f - ema_d) * p[h].y;
                        e[h].z = ema_d * e[h].z + (1.f - ema_d) * p[h].z;
                        e[h].w = ema_d * e[h].w + (1.f - ema_d) * p[h].w;
                        *reinterpret_cast<float4*>(ema + i + 4 * h) = e[h];
                    }
                }
            }
            // all-gather: the same 16 bytes to every rank's parameter buffer
            const uint4 raw = make_uint4(pack_bf16x2(p[0].x, p[0].y), pack_bf16x2(p[0].z, p[0].w),
                                         pack_bf16x2(p[1].x, p[1].y), pack_bf16x2(p[1].z, p[1].w));
            for (int j = 0; j < world; ++j) *reinterpret_cast<uint4*>(peers.param[j] + to_flat + i) = raw;
        }
    }
    // ---- completion: once every CTA's stores are out, tell every rank, wait for all
    __threadfence_system();
    if (last_cta(st.ticket)) {
        __threadfence_system();
        if (threadIdx.x < world) st_release_u32(peers.flags[threadIdx.x] + kFlagDone + rank, epoch);
        __syncthreads();
        if (threadIdx.x < world) {
            if (!wait_u32(st.flags_local + kFlagDone + threadIdx.x, epoch, st.spin_limit))
                record_error(st.status, kErrTimeoutDone);
        }
        __syncthreads();
        if (threadIdx.x == 0) *st.epoch = epoch + 1;  // next step (stream order publishes it)
    }
}

// Sum of a small fp32 vector over all ranks (num_boxes and other per-step
// scalars), one CTA, no host involvement.  Uses its own flag region.
__global__ void small_allreduce_kernel(DdpPeers peers, DdpState st, float* __restrict__ data, int n) {
    const uint32_t epoch = *st.small_epoch;
    const int world = peers.world, rank = peers.rank;
    // slots are double-buffered by epoch parity: a rank can only write the
    // buffer of epoch e+2 after every rank signalled e+1, i.e. finished reading e
    const int base = (epoch & 1u) * kDdpMaxWorld * kSmallMax;
    // publish my values to every rank's slot [rank]
    for (int i = threadIdx.x; i < n * world; i += blockDim.x) {
        const int j = i / n, k = i % n;
        peers.small[j][base + rank * kSmallMax + k] = data[k];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < world) st_release_u32(peers.flags[threadIdx.x] + kFlagSmall + rank, epoch);
    __shared__ int ok;
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if (threadIdx.x < world && !wait_u32(st.flags_local + kFlagSmall + threadIdx.x, epoch, st.spin_limit)) {
        record_error(st.status, kErrTimeoutSmall);
        ok = 0;
    }
    __syncthreads();
    if (ok) {
        for (int k = threadIdx.x; k < n; k += blockDim.x) {
            float s = 0.f;
            for (int j = 0; j < world; ++j) s += st.small_local[base + j * kSmallMax + k];
            data[k] = s;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *st.small_epoch = epoch + 1;
}

// Gradient all-reduce (optimizers that need every full gradient matrix, e.g. Muon): after the
// bucket reduce-scatters, each rank writes its reduced slices, rounded to bf16, into every rank's
// gradient buffer (16-byte P2P stores), then waits until every rank has delivered its slices and
// advances the step epoch.  Slices are given as (flat offset, length, shard-local offset).
struct SliceList {
    int64_t g_off[kDdpMaxBuckets], len[kDdpMaxBuckets], l_off[kDdpMaxBuckets];
    int n;
};

__global__ void __launch_bounds__(256) ddp_grad_allgather_kernel(DdpPeers peers, DdpState st, SliceList sl,
                                                                 const float* __restrict__ gshard) {
    const uint32_t epoch = *st.epoch;
    const int world = peers.world, rank = peers.rank;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int b = 0; b < sl.n; ++b) {
        const int64_t nvec = sl.len[b] / 8;
        for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
            float f[8];
            load8(gshard + sl.l_off[b] + 8 * v, f);
            const uint4 raw = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                                         pack_bf16x2(f[6], f[7]));
            for (int j = 0; j < world; ++j)
                *reinterpret_cast<uint4*>(const_cast<__nv_bfloat16*>(peers.grad[j]) + sl.g_off[b] + 8 * v) = raw;
        }
    }
    __threadfence_system();
    if (last_cta(st.ticket)) {
        __threadfence_system();
        if (threadIdx.x < world) st_release_u32(peers.flags[threadIdx.x] + kFlagDone + rank, epoch);
        __syncthreads();
        if (threadIdx.x < world) {
            if (!wait_u32(st.flags_local + kFlagDone + threadIdx.x, epoch, st.spin_limit))
                record_error(st.status, kErrTimeoutDone);
        }
        __syncthreads();
        if (threadIdx.x == 0) *st.epoch = epoch + 1;
    }
}

// Gather barrier: tell every rank (slot `rank` of region `base`) that this rank reached it with the
// current gather epoch, then wait for every rank's mark; `bump` advances the epoch afterwards.
__global__ void gather_barrier_kernel(DdpPeers peers, DdpState st, int base, int bump) {
    const uint32_t epoch = *st.gather_epoch;
    const int world = peers.world, rank = peers.rank;
    if (threadIdx.x < world) {
        __threadfence_system();
        st_release_u32(peers.flags[threadIdx.x] + base + rank, epoch);
    }
    __syncthreads();
    if (threadIdx.x < world && !wait_u32(st.flags_local + base + threadIdx.x, epoch, st.spin_limit))
        record_error(st.status, kErrTimeoutGather);
    __syncthreads();
    if (bump && threadIdx.x == 0) *st.gather_epoch = epoch + 1;
}

struct GatherPlan {
    int64_t off16[kDdpMaxWorld], len16[kDdpMaxWorld];
};

// every peer's staged payload (the start of its gradient buffer), 16-byte P2P loads
__global__ void __launch_bounds__(256) gather_copy_kernel(DdpPeers peers, uint4* __restrict__ out, GatherPlan plan) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int j = 0; j < peers.world; ++j) {
        const uint4* src = reinterpret_cast<const uint4*>(peers.grad[j]);
        uint4* dst = out + plan.off16[j];
        for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < plan.len16[j]; i += stride)
            dst[i] = ld_peer16(src + i);
    }
}

}  // namespace

cudaError_t launch_gather_bytes(const DdpPeers& peers, const DdpState& st, void* out, const int64_t* off16,
                                const int64_t* len16, cudaStream_t s) {
    if (peers.world < 1 || peers.world > kDdpMaxWorld || reinterpret_cast<uintptr_t>(out) % 16 != 0)
        return cudaErrorInvalidValue;
    GatherPlan plan{};
    int64_t total = 0;
    for (int j = 0; j < peers.world; ++j) {
        plan.off16[j] = off16[j];
        plan.len16[j] = len16[j];
        total += len16[j];
    }
    gather_barrier_kernel<<<1, 32, 0, s>>>(peers, st, kFlagGather, 0);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, num_sms() * 2)));
    gather_copy_kernel<<<blocks, 256, 0, s>>>(peers, static_cast<uint4*>(out), plan);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    gather_barrier_kernel<<<1, 32, 0, s>>>(peers, st, kFlagGatherDone, 1);
    return cudaGetLastError();
}

int ddp_rs_blocks(bool overlapped) { return overlapped ? 64 : num_sms() * 2; }

cudaError_t launch_ddp_grad_allgather(const DdpPeers& peers, const DdpState& st, const int64_t* g_off,
                                      const int64_t* len, const int64_t* l_off, int n, const float* gshard,
                                      cudaStream_t s) {
    if (n < 0 || n > kDdpMaxBuckets) return cudaErrorInvalidValue;
    SliceList sl{};
    sl.n = n;
    int64_t total = 0;
    for (int i = 0; i < n; ++i) {
        if (g_off[i] % 8 || len[i] % 8 || l_off[i] % 8) return cudaErrorInvalidValue;
        sl.g_off[i] = g_off[i];
        sl.len[i] = len[i];
        sl.l_off[i] = l_off[i];
        total += len[i];
    }
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((total / 8 + 255) / 256, num_sms() * 4)));
    ddp_grad_allgather_kernel<<<blocks, 256, 0, s>>>(peers, st, sl, gshard);
    return cudaGetLastError();
}

cudaError_t launch_ddp_rs(const DdpPeers& peers, const DdpState& st, int64_t g_off, int64_t len, float* gshard_at,
                          float* partials_b, int bucket, int blocks, cudaStream_t s) {
    if (len % 8 != 0 || g_off % 8 != 0 || peers.world < 1 || peers.world > kDdpMaxWorld || bucket < 0 ||
        bucket >= kDdpMaxBuckets || blocks < 1)
        return cudaErrorInvalidValue;
    const bool overlapped = blocks < num_sms();
    if (overlapped) {
        ddp_bucket_barrier_kernel<<<1, 32, 0, s>>>(peers, st, bucket);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    ddp_rs_kernel<<<blocks, 256, 0, s>>>(peers, st, g_off, len, gshard_at, partials_b, bucket, overlapped ? 0 : 1);
    return cudaGetLastError();
}

cudaError_t launch_ddp_publish(const DdpPeers& peers, const DdpState& st, const float* partials, int n,
                               cudaStream_t s) {
    ddp_publish_kernel<<<1, 32, 0, s>>>(peers, st, partials, n);
    return cudaGetLastError();
}

cudaError_t launch_ddp_update(const DdpPeers& peers, const DdpState& st, const ChunkDesc* chunks, const int64_t* gdelta,
                              int nchunks, const float* gshard, float* master, float* m, float* v, float* ema,
                              const GroupHyper* groups, const StepScalars* sc, int* flags, cudaStream_t s) {
    const int blocks = std::max(1, std::min(nchunks, num_sms() * 4));
    ddp_update_kernel<<<blocks, 256, 0, s>>>(peers, st, chunks, gdelta, nchunks, gshard, master, m, v, ema, groups, sc,
                                             flags);
    return cudaGetLastError();
}

cudaError_t launch_small_allreduce(const DdpPeers& peers, const DdpState& st, float* data, int n, cudaStream_t s) {
    if (n < 1 || n > kSmallMax) return cudaErrorInvalidValue;
    small_allreduce_kernel<<<1, 128, 0, s>>>(peers, st, data, n);
    return cudaGetLastError();
}

}  // namespace mmltk
