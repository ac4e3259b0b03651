// cuju-b200: crews, the unit of cooperation inside a warp.
//
// A crew is an aligned group of 1, 2, 4, 8, 16 or 32 lanes that advances one environment together.
// Every lane of a crew runs the environment's serial code with the same values (so nothing has to
// be broadcast), and the crew divides the wide loops of a tick between its lanes: the filters over
// ~1,500 animations, the sorts of candidate lists, the skeleton nodes of 25 humanoids, the
// per-frame physics precomputation. The kernels start every lane as a crew of one that owns its
// own environment; a branch that needs a wide loop can be handed to a larger crew (`crew_assist`
// in match_util.cuh).
//
// Each thread keeps its crew state in one byte of shared memory, written only by that thread:
//   bits 0-2  log2 of the crew width
//   bit  3    inside the body of a divided loop: the lane works alone on its share, and every
//             construct reached from there runs serially
//   bit  4    the lane's environment reached an iteration cap of GRF's arithmetic (a path GRF
//             leaves undefined); the step turns it into the environment's status
// Because no thread reads another thread's byte, changing a width needs no barrier; the barriers
// below only order the crew's memory accesses around a divided loop.
//
// The host build runs every construct serially (one environment per call, no crews).
#pragma once

#include "common.cuh"

namespace cb {

#if CB_DEVICE_PASS
CB_HD int crew_log2() { return crew_byte() & kCrewWidthBits; }
CB_HD int crew_width() { return 1 << crew_log2(); }
// This lane's place in its crew (0 for the crew's first lane).
CB_HD int crew_rank() { return lane_id() & (crew_width() - 1); }
CB_HD unsigned crew_mask() {
    const int w = crew_width();
    if (w == 32) return 0xffffffffu;
    return ((1u << w) - 1u) << (lane_id() & ~(w - 1));
}
// True where the code runs on one lane: a crew of one, or the body of a divided loop.
CB_HD bool crew_serial() {
    const uint8_t b = crew_byte();
    return (b & kCrewWidthBits) == 0 || (b & kCrewDividedBit) != 0;
}
// True where the lane is a crew of one that owns its environment (not inside a divided loop).
CB_HD bool crew_owns_env() { return (crew_byte() & (kCrewWidthBits | kCrewDividedBit)) == 0; }
CB_HD void crew_set(int log2w) { crew_byte() = (uint8_t)((crew_byte() & kCrewCapBit) | log2w); }
// Every kernel begins here: each lane a crew of one, no cap reached.
CB_HD void crew_start() { crew_byte() = 0; }
CB_HD void crew_sync() {
    if (!crew_serial()) __syncwarp(crew_mask());
}
// The lane that writes an environment's books: the crew's first lane.
CB_HD bool leader() { return crew_serial() || crew_rank() == 0; }

// Marks the lane as working alone on its share of a divided loop, and back.
struct CrewDivided {
    uint8_t saved;
    bool on;
    __device__ __forceinline__ explicit CrewDivided(bool enable = true) : saved(crew_byte()), on(enable) {
        if (on) crew_byte() = (uint8_t)(saved | kCrewDividedBit);
    }
    __device__ __forceinline__ ~CrewDivided() {
        if (on) crew_byte() = (uint8_t)((saved & ~kCrewCapBit) | (crew_byte() & kCrewCapBit));
    }
};

// Word-wise shuffle of a trivially copyable value from crew rank `src`.
template <class T>
__device__ __forceinline__ T crew_fetch(const T &v, int src) {
    static_assert(sizeof(T) % 4 == 0, "4-byte words");
    constexpr int W = (int)(sizeof(T) / 4);
    uint32_t in[W], out[W];
    memcpy(in, &v, sizeof(T));
    const unsigned m = crew_mask();
    const int w = crew_width();
#pragma unroll
    for (int k = 0; k < W; k++) out[k] = __shfl_sync(m, in[k], src, w);
    T r;
    memcpy(&r, out, sizeof(T));
    return r;
}
#else
CB_HD int crew_log2() { return 0; }
CB_HD void crew_set(int) {}
CB_HD int crew_width() { return 1; }
CB_HD int crew_rank() { return 0; }
CB_HD bool crew_serial() { return true; }
CB_HD bool crew_owns_env() { return true; }
CB_HD void crew_start() { crew_byte() = 0; }
CB_HD void crew_sync() {}
CB_HD bool leader() { return true; }
#endif

// body(i) for every i in [0, n), in no fixed order. Iterations share nothing and write only memory
// that every lane of the crew addresses (never a lane's locals).
template <class Body>
CB_HD void crew_for(int n, Body body) {
#if CB_DEVICE_PASS
    if (!crew_serial()) {
        const int w = crew_width();
        crew_sync();
        {
            CrewDivided divided;
            for (int i = crew_rank(); i < n; i += w) body(i);
        }
        crew_sync();
        return;
    }
#endif
    for (int i = 0; i < n; i++) body(i);
}

// emit(i) in increasing order of i for every i in [first, end) where pred(i) holds. A crew tests
// one index per lane at a time and then emits those that passed, in order, on every lane; so an
// emit may overwrite data at or below its own index (in-place compaction), and a predicate must
// write nothing that another index's predicate reads.
template <class Pred, class Emit>
CB_HD void crew_filter(int first, int end, Pred pred, Emit emit) {
#if CB_DEVICE_PASS
    if (!crew_serial()) {
        const int w = crew_width();
        const int rank = crew_rank();
        const unsigned mask = crew_mask();
        const int shift = lane_id() & ~(w - 1);
        for (int base = first; base < end; base += w) {
            crew_sync();
            bool pass;
            {
                CrewDivided divided;
                pass = base + rank < end && pred(base + rank);
            }
            unsigned bits = (__ballot_sync(mask, pass) & mask) >> shift;
            while (bits) {
                emit(base + __ffs(bits) - 1);
                bits &= bits - 1;
            }
        }
        return;
    }
#endif
    for (int i = first; i < end; i++)
        if (pred(i)) emit(i);
}

// body(i, pre(i)) for i in increasing order on every lane of the crew. `pre` is evaluated ahead,
// one index per lane, and must not read what `body` writes. T: trivially copyable, 4-byte words.
template <class T, class Pre, class Body>
CB_HD void crew_pipeline(int n, Pre pre, Body body) {
#if CB_DEVICE_PASS
    if (!crew_serial()) {
        const int w = crew_width();
        const int rank = crew_rank();
        for (int base = 0; base < n; base += w) {
            crew_sync();
            T mine;
            {
                CrewDivided divided;
                if (base + rank < n) mine = pre(base + rank);
            }
            const int count = n - base < w ? n - base : w;
            for (int src = 0; src < count; src++) body(base + src, crew_fetch(mine, src));
        }
        return;
    }
#endif
    for (int i = 0; i < n; i++) body(i, pre(i));
}

// out[i] = f(i) for i in [0, n) on every lane of the crew (`out` may be the lane's own array).
// V: 4 or 8 bytes.
template <class V, class F>
CB_HD void crew_map(int n, F f, V *out) {
#if CB_DEVICE_PASS
    if (!crew_serial()) {
        const int w = crew_width();
        const int rank = crew_rank();
        for (int base = 0; base < n; base += w) {
            crew_sync();
            V mine = V();
            {
                CrewDivided divided;
                if (base + rank < n) mine = f(base + rank);
            }
            const int count = n - base < w ? n - base : w;
            for (int src = 0; src < count; src++) out[base + src] = crew_fetch(mine, src);
        }
        return;
    }
#endif
    for (int i = 0; i < n; i++) out[i] = f(i);
}

// Copies `words` 4-byte words (or zero-fills them when `src` is null), divided between the lanes;
// both ranges in memory every lane of the crew addresses.
CB_HDNI void crew_copy_words(uint32_t *dst, const uint32_t *src, int words) {
#if CB_DEVICE_PASS
    if (!crew_serial()) {
        const int w = crew_width();
        crew_sync();
        for (int i = crew_rank(); i < words; i += w) dst[i] = src ? src[i] : 0u;
        crew_sync();
        return;
    }
#endif
    if (src) memcpy(dst, src, 4 * (size_t)words);
    else memset(dst, 0, 4 * (size_t)words);
}
template <class T>
CB_HD void crew_copy(T &dst, const T &src) {
    static_assert(sizeof(T) % 4 == 0, "words");
    crew_copy_words(reinterpret_cast<uint32_t *>(&dst), reinterpret_cast<const uint32_t *>(&src),
                    (int)(sizeof(T) / 4));
}

}  // namespace cb
