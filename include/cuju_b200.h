/* cuju-b200: the C-ABI of the B200 batch, a drop-in for the reference CUDA backend
 * (`libcuju_cuda.so`). Every entry point below has the name, arguments, meaning and error
 * convention of the reference function cited beside it, so the reference's Python loader binds
 * this library unchanged (set CUJU_CUDA_LIBRARY to its path).
 *
 * Conventions (cuju src/environment_api.h:3-6, 24-31): calls are synchronous unless noted; a
 * failure returns -1 or null, and `cuju_last_error` gives the message of the last failed call on
 * the calling thread. A `stream` is a CUDA stream, or null for the default stream. Buffers live in
 * device memory and never move until `cuju_environment_destroy`.
 */
#ifndef CUJU_B200_H
#define CUJU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cuju src/environment_api.h:47 */
#define CUJU_CONFIGURATION_VERSION 2

/* cuju src/environment_api.h:49-95 (field order fixed by python/cuju/_batch/library.py:156-187). */
typedef struct cuju_configuration {
    int version;
    const char *const *assets;
    int asset_count;
    const int *assignment;
    const char *animations;
    int environment_count;
    unsigned long long seed;
    int action_set;
    int observation;
    int checkpoints;
    int numpy_legacy;
    int auto_reset;
    int threads;
    int ticks_per_step;
    int smm_width, smm_height;
    int stack;
    const long long *fixed_seeds;
    const int *agent_counts;
    int episode_number;
    unsigned long long first_index;
    void *(*allocate)(size_t bytes, void *context);
    void (*release)(void *pointer, void *context);
    void *allocator_context;
    int pin_threads;
    int numa;
    int page_aligned;
} cuju_configuration;

/* environment_api.h:41 */ const char *cuju_last_error(void);
/* environment_api.h:44; returns "cuda" */ const char *cuju_backend(void);
/* environment_api.h:98 */ void *cuju_environment_create(const cuju_configuration *settings);
/* environment_api.h:161 */ int cuju_memory_estimate(const cuju_configuration *settings, unsigned long long *bytes);
/* environment_api.h:172 */ int cuju_local_memory_bytes(unsigned long long *bytes);
/* environment_api.h:186 */ unsigned long long cuju_environment_memory_bytes(void *environment);
/* environment_api.h:191 */ void cuju_environment_destroy(void *environment);
/* environment_api.h:195 */ int cuju_environment_count(void *environment);
/* environment_api.h:200; 0 on the GPU */ int cuju_environment_threads(void *environment);
/* environment_api.h:206 */ int cuju_environment_agents(void *environment, int *left, int *right);
/* environment_api.h:218 */ int cuju_environment_players(void *environment, int *left, int *right);
/* environment_api.h:229 */ int cuju_environment_set_difficulty(void *environment, const float *difficulty);
/* environment_api.h:240 */ void cuju_environment_difficulty(void *environment, float *difficulty);
/* environment_api.h:250 */ int cuju_environment_reset(void *environment, const unsigned int *seeds,
                                                        const int *reverse, void *stream);
/* environment_api.h:269 */ int cuju_environment_reset_masked(void *environment, const unsigned char *mask,
                                                               int mask_on_device, const int64_t *seeds,
                                                               const int *reverse, void *stream, int synchronize);
/* environment_api.h:287 */ int cuju_environment_reset_done(void *environment, void *stream);
/* environment_api.h:302; -2 for a host action outside [-n, n) */
int cuju_environment_step(void *environment, const int *actions, int on_device, void *stream, int synchronize);
/* environment_api.h:323 */ int cuju_environment_step_async(void *environment, const int *actions, int on_device,
                                                             void *stream);
/* environment_api.h:341 */ int cuju_environment_step_wait(void *environment);
/* environment_api.h:353 */ int cuju_environment_synchronize(void *environment, void *stream);
/* environment_api.h:367 */ const char *cuju_environment_get_state(void *environment, int index,
                                                                    unsigned long long *size, int *episode);
/* environment_api.h:392 */ int cuju_environment_set_state(void *environment, int index, const char *bytes,
                                                           unsigned long long size, const int *episode);
/* environment_api.h:410 */ int cuju_environment_set_stack(void *environment, int index, const char *name,
                                                           const void *frames, unsigned long long size);
/* environment_api.h:430; names simple115, final_simple115, reward, done, score_reward */
void *cuju_environment_buffer(void *environment, const char *name);
/* environment_api.h:449 */ const char *cuju_environment_raw_field(void *environment, int field, int *type,
                                                                    int *dimensions, unsigned long long *offset);
/* environment_api.h:470 */ int cuju_environment_episode(void *environment, int index, long long *values,
                                                         float *difficulty);
/* environment_api.h:519 */ const char *cuju_environment_scenario(void *environment, int bundle);
/* No reference counterpart: out[0] the kernels' per-thread local memory in bytes, out[1] their
 * registers per thread, out[2] the current per-thread stack limit. */
int cuju_b200_kernel_info(unsigned long long *out);
/* No reference counterpart. One step of a batch of at most 32 environments with actions already in
 * device memory of the current device, using a fixed 1.19 MiB device scratch array (room for 32
 * environments' sort keys) in place of the batch's own scratch. The success path allocates
 * nothing: no cudaMalloc/cudaFree, no host heap, no allocator callback. Asynchronous on `stream`
 * like cuju_environment_step_async; errors inside the step surface at the next
 * cuju_environment_synchronize. The first call on a device looks up the array's address with
 * cudaGetSymbolAddress while that device is current; make it before any stream capture. The
 * address is kept for the life of the process: after cudaDeviceReset (or anything else that
 * replaces the device's primary context) the kept address is stale, so do not call this entry
 * point again in that process. Nothing
 * in the array needs to start at zero (every sort writes what it reads). Calls that overlap in
 * time on one device (any stream, any batch) share the array and race: issue them one at a time.
 * Returns 0, or -1 with the reason in cuju_last_error (more than 32 environments, host or foreign
 * actions, a batch not yet reset, a CUDA error). */
int cuju_b200_environment_step_static(void *environment, const int *actions, void *stream);
/* No reference counterpart (the reference takes masked-reset seeds from the host only,
 * environment_api.h:263-271). A masked reset whose `mask` (uint8 [environments], nonzero = reset;
 * null = every environment) and `seeds` (int64 [environments]; negative draws the next seed of the
 * environment's generator, as -1 does in cuju_environment_reset_masked, and a value of 2^32 or
 * more keeps its low 32 bits; null = draw every seed) are both in device memory of the current
 * device. Nothing is checked or read on the host and nothing synchronises: the reset runs on
 * `stream` after the work before it, so a step and this reset can be captured in one CUDA graph.
 * A non-null `mask` is refused until every environment has started. Returns 0, or -1 with the
 * reason in cuju_last_error. */
int cuju_b200_environment_reset_masked_device(void *environment, const unsigned char *mask, const long long *seeds,
                                              void *stream);
/* No reference counterpart. How many lanes of a warp run each environment: 1 (each lane its own
 * environment; a warp's 32 lanes share the long branches in assist rounds), 2, 4, 8,
 * 16 or 32 (each environment a crew of that many lanes, which divide its wide loops), or 0 for the
 * default (the widest crews that keep the batch within four warps per SM: 1 lane for 16,384
 * environments on a 148-SM B200, 4 for 4,096, 32 for 592 or fewer). Results are
 * the same bits in every layout; only speed differs. Applies from the next launch. Returns 0, or -1
 * with the reason in cuju_last_error. */
int cuju_b200_environment_set_lanes(void *environment, int lanes);
/* state_api.h:21; 1 in `mask` at the padding bytes GRF saves uninitialized, 0 elsewhere */
int cuju_state_padding(const char *bytes, unsigned long long size, unsigned char *mask);
/* state_api.h:51 and :86 (the reference's in-memory state layout and a gather over it); this
 * backend's state lies differently in memory, so it returns null and -1 with a message */
const char *cuju_state_layout(unsigned long long *size);
int cuju_state_gather(const char *bytes, unsigned long long size, int frame, const unsigned long long *offsets,
                      const unsigned int *sizes, int count, unsigned char *out);

#ifdef __cplusplus
}
#endif

#endif /* CUJU_B200_H */
