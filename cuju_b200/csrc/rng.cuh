// cuju-b200: the two random number generators of a GRF environment.
//  * The match RNG: Boost.Random mt19937 plus its uniform float, whose state GRF stores in the
//    engine state as 2,512 bytes (624 words, a 64-bit index, min and max floats). cuju
//    include/cuju/rng.h:18-113.
//  * The episode seed generator: CPython's MT19937 `random` module, seeded as
//    `random.seed(seed * 2**32 + index)` and drawing `randint(0, 2000000000)`. cuju
//    include/cuju/batch/batch_core.h:262-341.
// Both are the published Mersenne Twister (Matsumoto & Nishimura 1998) with the two libraries'
// seeding rules.
#pragma once

#include "common.cuh"

namespace cb {

constexpr int kMtN = 624, kMtM = 397;

// View over the 2,512 serialized bytes (8-byte aligned inside the match).
struct MatchRng {
    uint8_t *b;
    CB_HD uint32_t *words() const { return reinterpret_cast<uint32_t *>(b); }
    CB_HD uint64_t index() const { return *reinterpret_cast<const uint64_t *>(b + 2496); }
    CB_HD void set_index(uint64_t v) { *reinterpret_cast<uint64_t *>(b + 2496) = v; }
    CB_HD float lo() const { return *reinterpret_cast<const float *>(b + 2504); }
    CB_HD float hi() const { return *reinterpret_cast<const float *>(b + 2508); }

    // Boost's seed(value): linear recurrence, then the normalisation that keeps only the top bit of
    // word 0 from it and maps an all-zero state to 1 << 31.
    CB_HDNI void seed(uint32_t v) {
        uint32_t *x = words();
        x[0] = v;
        for (int i = 1; i < kMtN; i++) x[i] = 1812433253u * (x[i - 1] ^ (x[i - 1] >> 30)) + (uint32_t)i;
        set_index(kMtN);
        const uint32_t upper = ~0u << 31, lower = ~upper, twist = 0x9908b0dfu;
        uint32_t y = x[kMtM - 1] ^ x[kMtN - 1];
        if (y & (1u << 31)) y = ((y ^ twist) << 1) | 1;
        else y = y << 1;
        x[0] = (x[0] & upper) | (y & lower);
        for (int i = 0; i < kMtN; i++)
            if (x[i] != 0) return;
        x[0] = 1u << 31;
    }
    CB_HDNI void twist() {
        uint32_t *x = words();
        const uint32_t upper = ~0u << 31, lower = ~upper, tm = 0x9908b0dfu;
        for (int i = 0; i < kMtN - kMtM; i++) {
            uint32_t y = (x[i] & upper) | (x[i + 1] & lower);
            x[i] = x[i + kMtM] ^ (y >> 1) ^ ((x[i + 1] & 1) * tm);
        }
        for (int i = kMtN - kMtM; i < kMtN - 1; i++) {
            uint32_t y = (x[i] & upper) | (x[i + 1] & lower);
            x[i] = x[i - (kMtN - kMtM)] ^ (y >> 1) ^ ((x[i + 1] & 1) * tm);
        }
        uint32_t y = (x[kMtN - 1] & upper) | (x[0] & lower);
        x[kMtN - 1] = x[kMtM - 1] ^ (y >> 1) ^ ((x[0] & 1) * tm);
        set_index(0);
    }
    CB_HD uint32_t next() {
        if (index() == kMtN) twist();
        uint64_t i = index();
        uint32_t z = words()[(int)i];
        set_index(i + 1);
        z ^= (z >> 11) & 0xffffffffu;
        z ^= (z << 7) & 0x9d2c5680u;
        z ^= (z << 15) & 0xefc60000u;
        z ^= (z >> 18);
        return z;
    }
    // Boost uniform_real<float>: Next()/2^32 in float, redrawn when it rounds up to the maximum.
    // A redraw happens about once in 2^25 draws for a range of [0, 1), so no match redraws 2^16
    // times in a row; the cap only ends the loop for a stored range where no draw can fall below
    // the maximum (equal or NaN bounds in corrupted state), which would otherwise never return; it
    // marks the environment (crew_note_cap), so the step ends in the unsupported-path status.
    CB_HD float uniform() {
        const float mn = lo(), mx = hi();
        float r = mn;
        for (unsigned redraws = 0; redraws < (1u << 16); redraws++) {
            float num = (float)(next() - 0u);
            float div = (float)(0xffffffffu - 0u) + 1;
            r = num / div * (mx - mn) + mn;
            if (r < mx) return r;
        }
        crew_note_cap();
        return r;
    }
};
CB_HD float random_in_range(uint8_t *rngBytes, float mn, float mx) {
    MatchRng g{rngBytes};
    float stretch = mx - mn;
    return mn + (g.uniform() * stretch);
}

// ---------------------------------------------------------------------------------------------
// CPython `random` (MT19937 with init_by_array).
struct EpisodeGen {
    uint32_t state[kMtN];
    int32_t next;  // kMtN when the state must turn over
};
CB_HDNI void episode_seed_words(EpisodeGen &g, const uint32_t *key, int n) {
    uint32_t *mt = g.state;
    mt[0] = 19650218u;
    for (int i = 1; i < kMtN; i++) mt[i] = 1812433253u * (mt[i - 1] ^ (mt[i - 1] >> 30)) + (uint32_t)i;
    int i = 1, j = 0;
    for (int k = kMtN > n ? kMtN : n; k; k--) {
        mt[i] = (mt[i] ^ ((mt[i - 1] ^ (mt[i - 1] >> 30)) * 1664525u)) + key[j] + (uint32_t)j;
        i++;
        j++;
        if (i >= kMtN) {
            mt[0] = mt[kMtN - 1];
            i = 1;
        }
        if (j >= n) j = 0;
    }
    for (int k = kMtN - 1; k; k--) {
        mt[i] = (mt[i] ^ ((mt[i - 1] ^ (mt[i - 1] >> 30)) * 1566083941u)) - (uint32_t)i;
        i++;
        if (i >= kMtN) {
            mt[0] = mt[kMtN - 1];
            i = 1;
        }
    }
    mt[0] = 0x80000000u;
    g.next = kMtN;
}
// random.seed(seed * 2**32 + index): the key is the 32-bit words of the integer, low first,
// trailing zero words dropped (at least one word).
CB_HD void episode_seed(EpisodeGen &g, uint64_t seed, uint32_t index) {
    const uint32_t w[3] = {index, (uint32_t)seed, (uint32_t)(seed >> 32)};
    int n = 3;
    while (n > 1 && w[n - 1] == 0) n--;
    episode_seed_words(g, w, n);
}
CB_HD uint32_t episode_word(EpisodeGen &g) {
    uint32_t *mt = g.state;
    if (g.next >= kMtN) {
        int k = 0;
        for (; k < kMtN - kMtM; k++) {
            uint32_t y = (mt[k] & 0x80000000u) | (mt[k + 1] & 0x7fffffffu);
            mt[k] = mt[k + kMtM] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        for (; k < kMtN - 1; k++) {
            uint32_t y = (mt[k] & 0x80000000u) | (mt[k + 1] & 0x7fffffffu);
            mt[k] = mt[k + kMtM - kMtN] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        uint32_t y = (mt[kMtN - 1] & 0x80000000u) | (mt[0] & 0x7fffffffu);
        mt[kMtN - 1] = mt[kMtM - 1] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        g.next = 0;
    }
    uint32_t y = mt[g.next++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}
// randint(0, 2000000000): 31-bit draws until one falls below 2000000001.
CB_HD uint32_t episode_draw_seed(EpisodeGen &g) {
    for (;;) {
        const uint32_t bits = episode_word(g) >> 1;
        if (bits < 2000000001u) return bits;
    }
}

}  // namespace cb
