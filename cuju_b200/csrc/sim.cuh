// cuju-b200: what a simulation function works on, and how a step reports failure.
#pragma once

#include "tables.cuh"

namespace cb {

// Errors a step can raise without trapping the device: recorded in the match's status word.
enum StepStatus : int32_t {
    kStatusOk = 0,
    kStatusUnsupported = 1,   // a path GRF leaves undefined
    kStatusOverflow = 2,      // a fixed-capacity list would overflow
};

// The sort scratch of one environment (global memory): bitonic pairs for a warp-wide sort, or
// the two key/position buffers of a merge sort when one lane owns the environment.
struct alignas(16) WarpScratch {
    double keys[2048];
    int16_t idx[2048];
    int16_t list[1536];
    double keys2[1536];
    int16_t idx2[1536];
};

// Everything a simulation function needs: the match, its context, the environment's sort scratch
// and its status word.
struct Sim {
    Match &w;
    const Context &ctx;
    WarpScratch *scratch;
    int32_t *status;
    CB_HD MatchState &m() const { return w.m; }
    CB_HD const AnimTables &T() const { return *ctx.anim; }
    CB_HD const Anim &A(int i) const { return ctx.anim->anims[i]; }
    CB_HD const AnimDerived &D(int i) const { return ctx.anim->derived[i]; }
    CB_HD bool fail(int32_t code) const {
        if (*status == kStatusOk) *status = code;
        return false;
    }
};

}  // namespace cb
