// cuju-b200: the launch interface between the host batch (api.cu) and the kernels (kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include "env.cuh"

namespace cb {

// The output kernel's block: two warps (64 environments).
constexpr int kThreadsPerBlock = 64;
// The step and reset kernels' blocks hold at most this many warps: one block per SM, whose warps
// move through a tick as a convoy (crew.cuh).
constexpr int kConvoyWarps = 4;

cudaError_t launch_step(const Batch &b, const int32_t *actions, cudaStream_t stream);
cudaError_t launch_reset(const Batch &b, const uint8_t *mask, const int64_t *seeds, const int32_t *reverse,
                         cudaStream_t stream);
cudaError_t launch_outputs(const Batch &b, const uint8_t *mask, cudaStream_t stream);
// The lanes per environment (log2) a batch of `count` environments runs with unless told otherwise.
cudaError_t default_crew_log2(int count, int *out);
// The largest per-thread local memory and register count of the kernels.
cudaError_t kernel_attributes(size_t *localBytes, int *registers);

// A fixed sort scratch in device memory (a file-scope array of kernels.cu) for the static-scratch
// step: room for kStaticScratchEnvironments environments, 32 x 38,912 B = 1.19 MiB per device.
constexpr int kStaticScratchEnvironments = 32;
constexpr int kStaticScratchDevices = 64;
// The array's address on the current device, looked up once per device (cudaGetSymbolAddress
// with that device current) and cached; allocates nothing.
cudaError_t static_scratch_address(WarpScratch **out);

}  // namespace cb
