// cuju-b200: one match per warp.
//
// Execution model: the 32 lanes of a warp run the serial part of a match redundantly (same
// values in every lane, so no broadcast is ever needed), and split the data-parallel loops of a
// tick (filters over ~1,500 animations, the 25 humanoids' skeleton nodes, sorts, per-frame
// physics precomputation) across lanes. A loop split across lanes is a "region": inside it the
// lanes diverge, so a helper reached from inside a region must run serially on its own lane.
// A per-warp flag in shared memory records whether the warp is inside a region.
// The host build (used for table preparation only) runs every loop serially.
#pragma once

#include "common.cuh"

namespace cb {

#if CB_DEVICE_PASS
CB_HD int lane_id() { return (int)(threadIdx.x & 31); }
__device__ __forceinline__ unsigned char &region_flag() {
    __shared__ unsigned char flags[32];
    return flags[threadIdx.x >> 5];
}
CB_HD void warp_begin() {
    if (lane_id() == 0) region_flag() = 0;
    __syncwarp();
}
CB_HD bool in_region() { return region_flag() != 0; }
// Set when each lane owns an environment of its own: every construct then runs serially on its
// lane, and per-environment scratch belongs to the lane.
CB_HD void lane_mode_begin() { region_flag() = 2; }
CB_HD bool lane_env() { return region_flag() == 2; }
// The lane that stores an environment's books: lane 0 of a warp that shares one environment, or
// every lane when each owns its own.
CB_HD bool leader() { return lane_env() || lane_id() == 0; }
CB_HD void region_enter() {
    __syncwarp();
    if (lane_id() == 0) region_flag() = 1;
    __syncwarp();
}
CB_HD void region_leave() {
    __syncwarp();
    if (lane_id() == 0) region_flag() = 0;
    __syncwarp();
}
// Lane and stride of a split loop at this point: the whole warp outside a region, this lane alone
// inside one.
CB_HD void split(bool &nested, int &lane, int &stride) {
    nested = in_region();
    lane = nested ? 0 : lane_id();
    stride = nested ? 1 : 32;
}
CB_HD void wsync() {
    if (!in_region()) __syncwarp();
}
#else
CB_HD int lane_id() { return 0; }
CB_HD void warp_begin() {}
CB_HD bool in_region() { return true; }
CB_HD void lane_mode_begin() {}
CB_HD bool lane_env() { return true; }
CB_HD bool leader() { return true; }
CB_HD void split(bool &nested, int &lane, int &stride) { nested = true; lane = 0; stride = 1; }
CB_HD void wsync() {}
#endif

// Calls `emit(i)` in increasing index order for every i in [first, end) with pred(i) true. The
// predicates of 32 consecutive indices are evaluated in parallel before their emits, so an emit
// may overwrite data at or below its own index (in-place compaction). Predicates write nothing
// another lane reads.
template <class Pred, class Emit>
CB_HD void par_filter(int first, int end, Pred pred, Emit emit) {
#if CB_DEVICE_PASS
    bool nested;
    int lane, stride;
    split(nested, lane, stride);
    for (int base = first; base < end; base += stride) {
        const int i = base + lane;
        if (!nested) region_enter();
        const bool keep = i < end && pred(i);
        if (!nested) region_leave();
        unsigned mask = nested ? (unsigned)keep : __ballot_sync(0xffffffffu, keep);
        while (mask) {
            emit(base + __ffs(mask) - 1);
            mask &= mask - 1;
        }
    }
#else
    for (int i = first; i < end; i++)
        if (pred(i)) emit(i);
#endif
}

// body(i) for every i in [0, n), in no fixed order; iterations share nothing and write only
// memory every lane addresses.
template <class Body>
CB_HD void par_for(int n, Body body) {
#if CB_DEVICE_PASS
    bool nested;
    int lane, stride;
    split(nested, lane, stride);
    if (!nested) region_enter();
    for (int i = lane; i < n; i += stride) body(i);
    if (!nested) region_leave();
#else
    for (int i = 0; i < n; i++) body(i);
#endif
}

// body(i, pre(i)) in index order on every lane; `pre` runs up to 32 iterations ahead in parallel
// and must not read what `body` writes. T is trivially copyable, a multiple of 4 bytes.
template <class T, class Pre, class Body>
CB_HD void par_pipeline(int n, Pre pre, Body body) {
#if CB_DEVICE_PASS
    static_assert(sizeof(T) % 4 == 0, "4-byte words");
    bool nested;
    int lane, stride;
    split(nested, lane, stride);
    for (int base = 0; base < n; base += stride) {
        T own;
        if (!nested) region_enter();
        if (base + lane < n) own = pre(base + lane);
        if (!nested) region_leave();
        constexpr int W = (int)(sizeof(T) / 4);
        uint32_t ow[W];
        memcpy(ow, &own, sizeof(T));
        const int cnt = n - base < stride ? n - base : stride;
        for (int src = 0; src < cnt; src++) {
            T v;
            if (nested) {
                v = own;
            } else {
                uint32_t w[W];
#pragma unroll
                for (int k = 0; k < W; k++) w[k] = __shfl_sync(0xffffffffu, ow[k], src);
                memcpy(&v, w, sizeof(T));
            }
            body(base + src, v);
        }
    }
#else
    for (int i = 0; i < n; i++) body(i, pre(i));
#endif
}

// Every lane receives out[i] = f(i) for i in [0, n). V is 4 or 8 bytes.
template <class V, class F>
CB_HD void par_map(int n, F f, V *out) {
#if CB_DEVICE_PASS
    bool nested;
    int lane, stride;
    split(nested, lane, stride);
    for (int base = 0; base < n; base += stride) {
        const int i = base + lane;
        if (!nested) region_enter();
        V v = i < n ? f(i) : V();
        if (!nested) region_leave();
        if (nested) {
            out[i] = v;
        } else {
            const int cnt = n - base < 32 ? n - base : 32;
            for (int src = 0; src < cnt; src++) out[base + src] = __shfl_sync(0xffffffffu, v, src);
        }
    }
#else
    for (int i = 0; i < n; i++) out[i] = f(i);
#endif
}

// Word copy (or zero fill when src is null) split across lanes; both in memory all lanes see.
CB_HDNI void par_copy_words(uint32_t *dst, const uint32_t *src, int words) {
#if CB_DEVICE_PASS
    wsync();
    bool nested;
    int lane, stride;
    split(nested, lane, stride);
    for (int i = lane; i < words; i += stride) dst[i] = src ? src[i] : 0u;
    wsync();
#else
    if (src) memcpy(dst, src, 4 * (size_t)words);
    else memset(dst, 0, 4 * (size_t)words);
#endif
}
template <class T>
CB_HD void par_copy(T &dst, const T &src) {
    static_assert(sizeof(T) % 4 == 0, "words");
    par_copy_words(reinterpret_cast<uint32_t *>(&dst), reinterpret_cast<const uint32_t *>(&src),
                   (int)(sizeof(T) / 4));
}

}  // namespace cb
