// cuju-b200: the batch kernels. Every lane starts as a crew of one that owns an environment and
// runs its whole step (crew.cuh); branches with wide loops are dealt to larger crews of the same
// warp (crew_assist). A warp advances 32 environments at once and a batch of 16,384 is resident in
// one wave. The host launches the kernels through the wrappers at the end, on the caller's stream.
#include <cuda_runtime.h>

#include <atomic>

#include "kernels.h"

namespace cb {

static_assert(kConvoyWarps * 32 <= kCrewSlots, "a block's threads each need a crew byte and a convoy key");

// A failed environment stops; the first failure code of the batch goes to `anyFail`.
__device__ __forceinline__ void report(const Batch &b, int e) {
    if (b.status[e] != kStatusOk) atomicCAS(b.anyFail, 0, b.status[e]);
}
__device__ __forceinline__ int env_index() { return (int)(blockIdx.x * blockDim.x + threadIdx.x); }
// The batch's warps spread evenly over the blocks (the first blocks take one warp more): warp w of
// block k runs environments 32 * (k * base + min(k, extra) + w) onwards. A warp past its block's
// share has none (count).
__device__ __forceinline__ int env_index_spread(int count) {
    const int warps = (count + 31) / 32, blocks = (int)gridDim.x, k = (int)blockIdx.x;
    const int base = warps / blocks, extra = warps % blocks;
    const int w = (int)(threadIdx.x >> 5);
    if (w >= base + (k < extra ? 1 : 0)) return count;
    return (k * base + (k < extra ? k : extra) + w) * 32 + lane_id();
}

// The environment of this thread within a launch of `count` environments: crews of one spread
// over the blocks, or one crew of 2^crewLog2 lanes per environment in blocks of kConvoyWarps warps.
__device__ __forceinline__ int env_index_for(const Batch &b, int count) {
    if (b.crewLog2 == 0) return env_index_spread(count);
    crew_set(b.crewLog2);
    return (int)((blockIdx.x * blockDim.x + threadIdx.x) >> b.crewLog2);
}

// A launch steps environments [first, first + count) of the batch (one wave, below).
__global__ void __launch_bounds__(kConvoyWarps * 32) step_kernel(Batch b, const int32_t *__restrict__ actions,
                                                                 int first, int count) {
    crew_start();
    const int local = env_index_for(b, count);
    const int e = first + local;
    const bool live = local < count && b.status[e] == kStatusOk;
    convoy_start(live);
    if (!live) return;
    step_environment(b, e, actions);
    settle_caps(b, e);
    report(b, e);
    convoy_leave();
}

// Resets every environment of [first, first + count) whose mask entry is set (all for a null mask).
__global__ void __launch_bounds__(kConvoyWarps * 32) reset_kernel(Batch b, const uint8_t *__restrict__ mask,
                                                                  const int64_t *__restrict__ seeds,
                                                                  const int32_t *__restrict__ reverse, int first,
                                                                  int count) {
    crew_start();
    const int local = env_index_for(b, count);
    const int e = first + local;
    const bool live = local < count && (!mask || mask[e]) && b.status[e] == kStatusOk;
    convoy_start(live);
    if (!live) return;
    reset_and_write(b, e, seeds, reverse);
    settle_caps(b, e);
    report(b, e);
    convoy_leave();
}

// Rewrites the outputs of the masked environments from their observations (after a state load).
__global__ void __launch_bounds__(kThreadsPerBlock) output_kernel(Batch b, const uint8_t *__restrict__ mask) {
    crew_start();
    const int e = env_index();
    if (e >= b.count || (mask && !mask[e])) return;
    write_env_outputs(b, e, false);
}

static unsigned grid_for(int count) {
    return (unsigned)((count + kThreadsPerBlock - 1) / kThreadsPerBlock);
}

// The SM count of the current device, looked up once per device.
static cudaError_t sm_count(int *out) {
    static std::atomic<int> cached[kStaticScratchDevices];
    int device = -1;
    cudaError_t rc = cudaGetDevice(&device);
    if (rc != cudaSuccess) return rc;
    if (device < 0 || device >= kStaticScratchDevices) return cudaErrorInvalidDevice;
    int n = cached[device].load(std::memory_order_acquire);
    if (n <= 0) {
        rc = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
        if (rc != cudaSuccess) return rc;
        cached[device].store(n, std::memory_order_release);
    }
    *out = n;
    return cudaSuccess;
}

// Convoy geometry: one block per SM while the batch has at most kConvoyWarps warps per SM (148
// blocks of 3 or 4 warps for 16,384 environments on a B200), blocks of kConvoyWarps warps beyond.
static cudaError_t convoy_geometry(int count, int crewLog2, dim3 &grid, dim3 &block) {
    int sms = 0;
    cudaError_t rc = sm_count(&sms);
    if (rc != cudaSuccess) return rc;
    if (crewLog2 > 0) {
        // Crews of 2^crewLog2 lanes per environment: one warp per block while the warps fit one per
        // SM (each SM's instruction cache serves one warp), kConvoyWarps warps per block beyond.
        const long long threads = (long long)count << crewLog2;
        const int perBlock = (threads + 31) / 32 <= sms ? 32 : kConvoyWarps * 32;
        grid = dim3((unsigned)((threads + perBlock - 1) / perBlock));
        block = dim3((unsigned)perBlock);
        return cudaSuccess;
    }
    const int warps = (count + 31) / 32;
    int blocks = (warps + kConvoyWarps - 1) / kConvoyWarps;
    if (blocks < sms) blocks = warps < sms ? warps : sms;
    grid = dim3((unsigned)blocks);
    block = dim3((unsigned)(32 * ((warps + blocks - 1) / blocks)));
    return cudaSuccess;
}

// Waves: a batch larger than kConvoyWarps warps on every SM runs as equal waves of at most that
// many environments, one launch after another on the stream. More warps per SM than that only
// make the SM's warps evict each other's instructions (65,536 environments in one launch ran at
// 3.2 s a step on a B200, in four launches of 16,384 at 2.2 s), and environments do not depend on
// each other, so the split changes no result.
static cudaError_t wave_size(int count, int crewLog2, int *out) {
    int sms = 0;
    cudaError_t rc = sm_count(&sms);
    if (rc != cudaSuccess) return rc;
    const long long full = ((long long)sms * kConvoyWarps * 32) >> crewLog2;
    if (count <= full || full <= 0) {
        *out = count;
        return cudaSuccess;
    }
    const long long waves = (count + full - 1) / full;
    *out = (int)((count + waves - 1) / waves);
    return cudaSuccess;
}

cudaError_t launch_step(const Batch &b, const int32_t *actions, cudaStream_t stream) {
    int wave = 0;
    cudaError_t rc = wave_size(b.count, b.crewLog2, &wave);
    for (int first = 0; rc == cudaSuccess && first < b.count; first += wave) {
        const int count = b.count - first < wave ? b.count - first : wave;
        dim3 grid, block;
        rc = convoy_geometry(count, b.crewLog2, grid, block);
        if (rc != cudaSuccess) return rc;
        step_kernel<<<grid, block, 0, stream>>>(b, actions, first, count);
        rc = cudaGetLastError();
    }
    return rc;
}
cudaError_t launch_reset(const Batch &b, const uint8_t *mask, const int64_t *seeds, const int32_t *reverse,
                         cudaStream_t stream) {
    int wave = 0;
    cudaError_t rc = wave_size(b.count, b.crewLog2, &wave);
    for (int first = 0; rc == cudaSuccess && first < b.count; first += wave) {
        const int count = b.count - first < wave ? b.count - first : wave;
        dim3 grid, block;
        rc = convoy_geometry(count, b.crewLog2, grid, block);
        if (rc != cudaSuccess) return rc;
        reset_kernel<<<grid, block, 0, stream>>>(b, mask, seeds, reverse, first, count);
        rc = cudaGetLastError();
    }
    return rc;
}
cudaError_t launch_outputs(const Batch &b, const uint8_t *mask, cudaStream_t stream) {
    output_kernel<<<grid_for(b.count), kThreadsPerBlock, 0, stream>>>(b, mask);
    return cudaGetLastError();
}
// The static-scratch step's sort scratch. Nothing in it needs to start at zero: every sort writes
// the keys and positions it reads.
static __device__ __align__(256) WarpScratch staticScratch[kStaticScratchEnvironments];

cudaError_t static_scratch_address(WarpScratch **out) {
    static std::atomic<WarpScratch *> cached[kStaticScratchDevices];
    int device = -1;
    cudaError_t rc = cudaGetDevice(&device);
    if (rc != cudaSuccess) return rc;
    if (device < 0 || device >= kStaticScratchDevices) return cudaErrorInvalidDevice;
    WarpScratch *p = cached[device].load(std::memory_order_acquire);
    if (!p) {
        void *address = nullptr;
        rc = cudaGetSymbolAddress(&address, staticScratch);
        if (rc != cudaSuccess) return rc;
        p = static_cast<WarpScratch *>(address);
        cached[device].store(p, std::memory_order_release);
    }
    *out = p;
    return cudaSuccess;
}

cudaError_t kernel_attributes(size_t *localBytes, int *registers) {
    cudaFuncAttributes a;
    cudaError_t rc = cudaFuncGetAttributes(&a, step_kernel);
    if (rc != cudaSuccess) return rc;
    size_t lb = a.localSizeBytes;
    int regs = a.numRegs;
    rc = cudaFuncGetAttributes(&a, reset_kernel);
    if (rc != cudaSuccess) return rc;
    if (a.localSizeBytes > lb) lb = a.localSizeBytes;
    if (a.numRegs > regs) regs = a.numRegs;
    *localBytes = lb;
    *registers = regs;
    return cudaSuccess;
}

}  // namespace cb

namespace cb {
cudaError_t default_crew_log2(int count, int *out) {
    int sms = 0;
    cudaError_t rc = sm_count(&sms);
    if (rc != cudaSuccess) return rc;
    // The widest crews that keep the batch within kConvoyWarps warps per SM: a lane per environment
    // for 16,384 environments on 148 SMs, 4 lanes for 4,096, a warp each for 592 or fewer. Beyond
    // about four warps per SM the instruction cache, not the lanes, limits an SM, so wider crews
    // there only add redundant lanes.
    int log2 = 0;
    while (log2 < 5 && ((long long)count << (log2 + 1)) <= (long long)sms * kConvoyWarps * 32) log2++;
    *out = log2;
    return cudaSuccess;
}
}  // namespace cb
