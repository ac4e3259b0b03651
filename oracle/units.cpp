// Test infrastructure only: entry points into the reference headers, compiled with them from the
// reference sources into oracle/_ref/liboracle_units.so. Parity tests use them as the checker;
// nothing in the product loads this library.
//
// oracle_state_paths: the field path, saved position and size of every field of a GRF state, as
// the reference's own codec visits them (cuju include/cuju/state/archive.h:76-110 layout mode,
// include/cuju/simulation/state_io.h:20-60 load), so a byte offset where two states differ names
// the field that differs.
#include <memory>
#include <string>
#include <vector>

#include "cuju/simulation/state_io.h"

extern "C" __attribute__((visibility("default"))) const char *oracle_state_paths(const char *bytes,
                                                                               unsigned long long size,
                                                                               unsigned long long *outSize) {
    static thread_local std::string text;
    text.clear();
    try {
        auto world = std::make_unique<cuju::simulation::World>();
        cuju::simulation::StateCodec codec;
        if (!codec.Load(std::string(bytes, size), *world)) {
            text = "error: the state does not load";
            *outSize = text.size();
            return text.c_str();
        }
        std::vector<cuju::state::LayoutEntry> layout;
        cuju::state::Archive archive = cuju::state::Archive::Saver();
        archive.layout = &layout;
        archive.layoutBase = &world->serialized;
        archive.layoutStorage = false;
        cuju::state::ProcessEnvironmentState(archive, world->serialized, codec.freeControllerCount);
        for (const cuju::state::LayoutEntry &e : layout)
            text += std::to_string(e.position) + "\t" + std::to_string(e.size) + "\t" + e.path + "\n";
        *outSize = text.size();
        return text.c_str();
    } catch (const std::exception &e) {
        text = std::string("error: ") + e.what();
        *outSize = text.size();
        return text.c_str();
    }
}

// oracle_hungarian: the reference's assignment solver (cuju include/cuju/simulation/team_ai.h:250)
// on a row-major `size` x `size` cost matrix; returns its total and writes the column of each row.
#include "cuju/simulation/team_ai.h"
extern "C" __attribute__((visibility("default"))) int oracle_hungarian(const int *cost, int size, int *columns) {
    cuju::simulation::HungarianMatrix m;
    for (int i = 0; i < size * size; i++) m.push_back(cost[i]);
    cuju::simulation::HungarianRow cols;
    const int total = cuju::simulation::HungarianSolve(m, size, cols);
    if (total != -1)
        for (int i = 0; i < size; i++) columns[i] = cols[i];
    return total;
}

// The reference's range wrap (cuju include/cuju/math_utilities.h:33, GRF's ModulateIntoRange).
// Callers pass only values on which its loops end (|value| below 2^27 for a span of 2*pi).
#include "cuju/math_utilities.h"

extern "C" __attribute__((visibility("default"))) float oracle_modulate_into_range(float min, float max,
                                                                                  float value) {
    return cuju::ModulateIntoRange(min, max, value);
}

// oracle_libm: the reference's restatements of glibc's math functions (cuju include/cuju/libm/*.h),
// `n` evaluations of function `which` on x (and y for the two-argument ones), each result widened
// to double. Functions: 0 sinf, 1 cosf, 2 powf, 3 acosf, 4 asinf, 5 atanf, 6 atan2f, 7 sin, 8 cos,
// 9 acos, 10 pow; 11, 12 and 13 are sinf, cosf and powf again (the checks of the library's
// sine-and-cosine pair and of its positive-base power).
#include "cuju/libm/acos_double.h"
#include "cuju/libm/asinf.h"
#include "cuju/libm/inverse_trigonometric_float.h"
#include "cuju/libm/pow.h"
#include "cuju/libm/powf.h"
#include "cuju/libm/sin_double.h"
#include "cuju/libm/sincosf.h"

extern "C" __attribute__((visibility("default"))) int oracle_libm(int which, const double *x, const double *y,
                                                                 double *out, int n) {
    for (int i = 0; i < n; i++) {
        const float xf = (float)x[i], yf = (float)y[i];
        switch (which) {
            case 0: out[i] = cuju::libm::sinf(xf); break;
            case 1: out[i] = cuju::libm::cosf(xf); break;
            case 2: out[i] = cuju::libm::powf(xf, yf); break;
            case 3: out[i] = cuju::libm::acosf(xf); break;
            case 4: out[i] = cuju::libm::asinf(xf); break;
            case 5: out[i] = cuju::libm::atanf(xf); break;
            case 6: out[i] = cuju::libm::atan2f(yf, xf); break;
            case 7: out[i] = cuju::libm::sin(x[i]); break;
            case 8: out[i] = cuju::libm::cos(x[i]); break;
            case 9: out[i] = cuju::libm::acos(x[i]); break;
            case 10: out[i] = cuju::libm::pow(x[i], y[i]); break;
            case 11: out[i] = cuju::libm::sinf(xf); break;
            case 12: out[i] = cuju::libm::cosf(xf); break;
            case 13: out[i] = cuju::libm::powf(xf, yf); break;
            default: return -1;
        }
    }
    return 0;
}
