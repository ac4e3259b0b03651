// cuju-b200: the batch kernels. Every lane starts as a crew of one that owns an environment and
// runs its whole step (crew.cuh); branches with wide loops are dealt to larger crews of the same
// warp (crew_assist). A warp advances 32 environments at once and a batch of 16,384 is resident in
// one wave. The host launches the kernels through the wrappers at the end, on the caller's stream.
#include <cuda_runtime.h>

#include <atomic>

#include "kernels.h"

namespace cb {

// A failed environment stops; the first failure code of the batch goes to `anyFail`.
__device__ __forceinline__ void report(const Batch &b, int e) {
    if (b.status[e] != kStatusOk) atomicCAS(b.anyFail, 0, b.status[e]);
}
__device__ __forceinline__ int env_index() { return (int)(blockIdx.x * blockDim.x + threadIdx.x); }

__global__ void __launch_bounds__(kThreadsPerBlock) step_kernel(Batch b, const int32_t *__restrict__ actions) {
    crew_start();
    const int e = env_index();
    if (e >= b.count || b.status[e] != kStatusOk) return;
    step_environment(b, e, actions);
    settle_caps(b, e);
    report(b, e);
}

// Resets every environment whose mask entry is set (all for a null mask).
__global__ void __launch_bounds__(kThreadsPerBlock) reset_kernel(Batch b, const uint8_t *__restrict__ mask,
                                                                 const int64_t *__restrict__ seeds,
                                                                 const int32_t *__restrict__ reverse) {
    crew_start();
    const int e = env_index();
    if (e >= b.count || (mask && !mask[e]) || b.status[e] != kStatusOk) return;
    reset_and_write(b, e, seeds, reverse);
    settle_caps(b, e);
    report(b, e);
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

cudaError_t launch_step(const Batch &b, const int32_t *actions, cudaStream_t stream) {
    step_kernel<<<grid_for(b.count), kThreadsPerBlock, 0, stream>>>(b, actions);
    return cudaGetLastError();
}
cudaError_t launch_reset(const Batch &b, const uint8_t *mask, const int64_t *seeds, const int32_t *reverse,
                         cudaStream_t stream) {
    reset_kernel<<<grid_for(b.count), kThreadsPerBlock, 0, stream>>>(b, mask, seeds, reverse);
    return cudaGetLastError();
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
