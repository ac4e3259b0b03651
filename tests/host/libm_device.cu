// Test infrastructure: the library's math functions (cuju_b200/csrc/libm.cuh) evaluated on a B200,
// for the per-function check against the reference's restatements (tests/test_gpu_libm.py). Built
// by that test with the library's own floating-point flags; nothing in the product loads it.
#include <cuda_runtime.h>

#include "libm_eval.cuh"

__global__ void libm_kernel(int which, const double *x, const double *y, double *out, int n) {
    const int i = (int)(blockIdx.x * blockDim.x + threadIdx.x);
    if (i < n) out[i] = libm_eval(which, x[i], y[i]);
}

// Host arrays in and out; returns 0, or the CUDA error code.
extern "C" __attribute__((visibility("default"))) int libm_device_eval(int which, const double *x, const double *y,
                                                                      double *out, int n) {
    double *d = nullptr;
    const size_t bytes = sizeof(double) * (size_t)n;
    cudaError_t rc = cudaMalloc(&d, 3 * bytes);
    if (rc != cudaSuccess) return (int)rc;
    if ((rc = cudaMemcpy(d, x, bytes, cudaMemcpyHostToDevice)) == cudaSuccess &&
        (rc = cudaMemcpy(d + n, y, bytes, cudaMemcpyHostToDevice)) == cudaSuccess) {
        libm_kernel<<<(n + 127) / 128, 128>>>(which, d, d + n, d + 2 * (size_t)n, n);
        rc = cudaGetLastError();
        if (rc == cudaSuccess) rc = cudaMemcpy(out, d + 2 * (size_t)n, bytes, cudaMemcpyDeviceToHost);
    }
    cudaFree(d);
    return (int)rc;
}
