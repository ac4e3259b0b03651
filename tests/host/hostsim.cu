// Test infrastructure, not part of the library: the library's C-ABI (api.cu) and simulation
// headers compiled for the host, with host memory standing in for device memory and each kernel
// replaced by a serial loop over the environments. It lets CPU-only tests run long golden matches
// through the same simulation source the kernels compile, at host speed. Built by
// tests/test_host_long.py into a temporary directory; nothing in the product loads it.
#include <cuda_runtime.h>
#include <cstdlib>
#include <cstring>
#include <cstdio>

static cudaError_t hs_malloc(void **p, size_t n) { *p = aligned_alloc(256, (n + 255) & ~(size_t)255); if (*p) memset(*p, 0, (n + 255) & ~(size_t)255); return *p ? cudaSuccess : cudaErrorMemoryAllocation; }
static cudaError_t hs_memset(void *p, int v, size_t n) { memset(p, v, n); return cudaSuccess; }
static cudaError_t hs_free(void *p) { free(p); return cudaSuccess; }
static cudaError_t hs_memcpy(void *d, const void *s, size_t n, cudaMemcpyKind) { memmove(d, s, n); return cudaSuccess; }
static cudaError_t hs_memcpy_async(void *d, const void *s, size_t n, cudaMemcpyKind, cudaStream_t) { memmove(d, s, n); return cudaSuccess; }
static cudaError_t hs_ok0() { return cudaSuccess; }
static cudaError_t hs_ok1(cudaStream_t) { return cudaSuccess; }
static cudaError_t hs_get_limit(size_t *v, cudaLimit) { *v = 0; return cudaSuccess; }
static cudaError_t hs_set_limit(cudaLimit, size_t) { return cudaSuccess; }
static cudaError_t hs_get_device(int *d) { *d = 0; return cudaSuccess; }
#define cudaMalloc(p, n) hs_malloc((void **)(p), n)
#define cudaMemset hs_memset
#define cudaFree hs_free
#define cudaMemcpy hs_memcpy
#define cudaMemcpyAsync hs_memcpy_async
#define cudaDeviceSynchronize hs_ok0
#define cudaStreamSynchronize hs_ok1
#define cudaDeviceGetLimit hs_get_limit
#define cudaDeviceSetLimit hs_set_limit
#define cudaGetDevice hs_get_device
#define cuju_backend cuju_backend_product
#include "api.cu"
#undef cuju_backend

namespace cb {
cudaError_t launch_step(const Batch &b, const int32_t *actions, cudaStream_t) {
    for (int e = 0; e < b.count; e++) {
        if (b.status[e]) continue;
        crew_start();
        step_environment(b, e, actions);
        settle_caps(b, e);
        if (b.status[e] && !*b.anyFail) { *b.anyFail = b.status[e]; fprintf(stderr, "env %d failed %d\n", e, b.status[e]); }
    }
    return cudaSuccess;
}
cudaError_t launch_reset(const Batch &b, const uint8_t *mask, const int64_t *seeds, const int32_t *reverse, cudaStream_t) {
    for (int e = 0; e < b.count; e++) {
        if (mask && !mask[e]) continue;
        if (b.status[e]) continue;
        crew_start();
        reset_and_write(b, e, seeds, reverse);
        settle_caps(b, e);
        if (b.status[e] && !*b.anyFail) { *b.anyFail = b.status[e]; fprintf(stderr, "env %d failed %d\n", e, b.status[e]); }
    }
    return cudaSuccess;
}
cudaError_t launch_outputs(const Batch &b, const uint8_t *mask, cudaStream_t) {
    for (int e = 0; e < b.count; e++) if (!mask || mask[e]) write_env_outputs(b, e, false);
    return cudaSuccess;
}
cudaError_t kernel_attributes(size_t *l, int *r) { *l = 0; *r = 0; return cudaSuccess; }
cudaError_t default_crew_log2(int, int *out) { *out = 0; return cudaSuccess; }
cudaError_t static_scratch_address(WarpScratch **out) { *out = nullptr; return cudaErrorNotSupported; }
}
extern "C" __attribute__((visibility("default"))) const char *cuju_backend() { return "cpu"; }

#include "libm_eval.cuh"

#include <random>

// The touch's repeated ball prediction: for `trials` seeded balls (on the ground, in flight, at
// rest, against a post, in the goal), the ball after ball_recalc run twice and after ball_recalc
// then ball_recalc_again, from an empty prediction cache as ball_touch leaves it. Odd trials also
// set the first run's 20 ms entry to its 10 ms entry in both copies before the second call, so
// that the second call takes its cached shift (a ball that does not move between 10 and 20 ms,
// which real flights hardly produce). Returns the number of trials whose balls differ in any
// byte, and counts the trials whose second call shifted (`shifted`).
extern "C" __attribute__((visibility("default"))) int hostsim_check_recalc_again(unsigned seed, int trials,
                                                                                int *shifted) {
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> u(-1.0f, 1.0f);
    auto *a = static_cast<cb::Match *>(calloc(1, sizeof(cb::Match)));
    auto *b = static_cast<cb::Match *>(calloc(1, sizeof(cb::Match)));
    int bad = 0;
    *shifted = 0;
    for (int t = 0; t < trials; t++) {
        memset(a, 0, sizeof(cb::Match));
        cb::Ball &ball = a->m.ball;
        const int kind = (t / 2) % 5;
        ball.positionBuffer = cb::Vec3(55.0f * u(rng), 36.0f * u(rng), 0.11f);
        if (kind == 1) ball.positionBuffer.c[2] = 0.11f + 4.0f * (u(rng) + 1.0f);
        if (kind == 3) ball.positionBuffer = cb::Vec3(54.9f + 0.1f * u(rng), 3.7f + 0.05f * u(rng), 0.5f + u(rng));
        if (kind == 4) ball.positionBuffer = cb::Vec3(56.0f + u(rng), 2.0f * u(rng), 0.5f + 0.4f * u(rng));
        ball.momentum = kind == 2 ? cb::Vec3(0.0f) : cb::Vec3(25.0f * u(rng), 25.0f * u(rng), 8.0f * u(rng));
        const float s = 0.01f * u(rng);
        ball.rotationPerMs = kind == 2 ? cb::Quat::identity() : cb::Quat(s, -s, 0.5f * s, 1.0f).normalized();
        ball.orientationBuffer = cb::Quat(0.1f * u(rng), 0.1f * u(rng), 0.1f * u(rng), 1.0f).normalized();
        ball.validPredictions = 0;
        a->m.ballIsInGoal = kind == 4;
        cb::ball_recalc(*a);
        if (t % 2) a->m.ball.predictions[2] = a->m.ball.predictions[1];
        memcpy(b, a, sizeof(cb::Match));
        cb::ball_recalc(*a);
        if (b->m.ball.validPredictions > 0 && b->m.ball.predictions[2] == b->m.ball.predictions[1]) (*shifted)++;
        cb::ball_recalc_again(b->m.ball);
        if (memcmp(&a->m.ball, &b->m.ball, sizeof(cb::Ball)) != 0) bad++;
    }
    free(a);
    free(b);
    return bad;
}

// The library's math functions on the host, for the per-function check against the reference's
// restatements (tests/test_libm.py; numbering of libm_eval.cuh).
extern "C" __attribute__((visibility("default"))) int hostsim_libm(int which, const double *x, const double *y,
                                                                  double *out, int n) {
    for (int i = 0; i < n; i++) out[i] = libm_eval(which, x[i], y[i]);
    return 0;
}

// The device code's range wrap, for a unit check against the reference's (tests/test_host_api.py).
extern "C" __attribute__((visibility("default"))) float hostsim_wrap_range(float lo, float hi, float v) {
    return cb::wrap_range(lo, hi, v);
}
