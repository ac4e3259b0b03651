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
