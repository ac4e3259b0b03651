// cuju-b200: the C-ABI of the batch, a drop-in for the reference's `libcuju_cuda.so` (the
// `cuju_*` functions and `cuju_configuration` version 2 of cuju src/environment_api.h). The host
// keeps the books (bundles, variants, seeds, checks); every reset and step runs on the device.
// Errors: -1 or null with the message in a thread-local string (`cuju_last_error`), -2 for a host
// action out of range, as the reference does.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/cuju_b200.h"
#include "assets.h"
#include "kernels.h"

namespace cb {
namespace host {

struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
static void check(cudaError_t rc, const char *what) {
    if (rc != cudaSuccess) throw CudaError(std::string("cuda error in ") + what + ": " + cudaGetErrorString(rc));
}

// Optional caller-provided device allocator (the reference's allocate/release callbacks).
struct Allocator {
    void *(*allocate)(size_t, void *) = nullptr;
    void (*release)(void *, void *) = nullptr;
    void *context = nullptr;
    size_t bytes = 0;
    unsigned long long *estimate = nullptr;  // counting only: no memory is taken
    std::vector<void *> blocks;

    void *get(size_t n) {
        if (n == 0) n = 1;
        n = (n + 255) & ~(size_t)255;
        bytes += n;
        if (estimate) {
            *estimate += n;
            return nullptr;
        }
        void *p = nullptr;
        if (allocate) {
            p = allocate(n, context);
            if (!p) throw std::runtime_error("the allocator has no device memory for " + std::to_string(n) + " bytes");
        } else {
            check(cudaMalloc(&p, n), "cudaMalloc");
        }
        check(cudaMemset(p, 0, n), "cudaMemset");
        blocks.push_back(p);
        return p;
    }
    ~Allocator() {
        if (!blocks.empty()) cudaDeviceSynchronize();
        for (void *p : blocks) {
            if (release) release(p, context);
            else cudaFree(p);
        }
    }
};

struct Config {
    std::vector<std::string> assets;
    std::vector<int32_t> assignment;
    std::string animations;
    int count = 1;
    uint64_t seed = 0;
    int actionSet = 0;
    int observation = kObsSimple115v2;
    bool checkpoints = false, numpyLegacy = true, autoReset = true;
    int ticksPerStep = 10;
    int smmWidth = 96, smmHeight = 72;
    int stack = 1;
    std::vector<int64_t> fixedSeeds;
    std::vector<int32_t> agentCounts;
    int episodeNumber = 0;
    int64_t firstIndex = 0;
    void *(*allocate)(size_t, void *) = nullptr;
    void (*release)(void *, void *) = nullptr;
    void *allocatorContext = nullptr;
};

// batch_core.h:121 (MakeRawLayout): the shape of each raw array after the agent axis, and its
// place in one buffer (each array starting at a multiple of 256 bytes).
inline RawLayout make_raw_layout(size_t outputs, int players, int sticky) {
    RawLayout lay{};
    lay.players = players;
    int shape[kRawFields][3] = {{kRawF32, 3, 0}, {kRawF32, 3, 0}, {kRawF32, 3, 0}, {kRawI32, 0, 0}, {kRawI32, 0, 0}};
    const int team[6][3] = {{kRawF32, players, 2}, {kRawF32, players, 2}, {kRawF32, players, 0},
                            {kRawBool, players, 0}, {kRawBool, players, 0}, {kRawI32, players, 0}};
    for (int t = 0; t < 2; t++)
        for (int f = 0; f < 6; f++)
            for (int k = 0; k < 3; k++) shape[kRawLeftTeam + 6 * t + f][k] = team[f][k];
    const int tail[6][3] = {{kRawI32, 2, 0}, {kRawI32, 0, 0}, {kRawI32, 0, 0},
                            {kRawI32, 0, 0}, {kRawI32, 0, 0}, {kRawU8, sticky, 0}};
    for (int f = 0; f < 6; f++)
        for (int k = 0; k < 3; k++) shape[kRawScore + f][k] = tail[f][k];
    uint64_t offset = 0;
    for (int f = 0; f < kRawFields; f++) {
        RawArray &a = lay.arrays[f];
        a.type = shape[f][0];
        a.dims[0] = shape[f][1];
        a.dims[1] = shape[f][2];
        a.elements = (a.dims[0] ? a.dims[0] : 1) * (a.dims[1] ? a.dims[1] : 1);
        a.offset = offset;
        const int size = a.type == kRawF32 || a.type == kRawI32 ? 4 : 1;
        offset += (outputs * a.elements * size + 255) / 256 * 256;
    }
    lay.bytes = offset;
    return lay;
}

class BatchEnv {
public:
    Allocator mem;
    Config cfg;
    std::vector<Assets> bundles;
    std::unique_ptr<AnimStore> store;
    Batch b{};
    std::vector<EnvSlot> hostSlots;
    std::vector<float> hostDifficulty;
    std::vector<bool> started;
    int unstarted = 0;
    int players = 0;
    std::vector<Variant> hostVariants;
    int32_t *actionsDev = nullptr;
    uint8_t *maskDev = nullptr;
    int64_t *seedsDev = nullptr;
    int32_t *reverseDev = nullptr;
    uint8_t *outputMaskDev = nullptr;

    template <class T>
    T *alloc(size_t n) {
        return static_cast<T *>(mem.get(sizeof(T) * n));
    }
    template <class T>
    T *upload(const T *src, size_t n) {
        T *d = alloc<T>(n);
        if (d && n) check(cudaMemcpy(d, src, sizeof(T) * n, cudaMemcpyHostToDevice), "upload");
        return d;
    }
    template <class T>
    T *upload(const std::vector<T> &v) {
        return upload(v.data(), v.size());
    }

    explicit BatchEnv(const Config &c, unsigned long long *estimate) : cfg(c) {
        mem.estimate = estimate;
        mem.allocate = c.allocate;
        mem.release = c.release;
        mem.context = c.allocatorContext;
        if ((c.observation & kObsSimple115) && (c.observation & kObsSimple115v2))
            throw std::invalid_argument("simple115 and simple115v2 are exclusive");
        if (!(c.observation & (kObsSimple115 | kObsSimple115v2 | kObsSmm | kObsRaw)))
            throw std::invalid_argument("expected the simple115, simple115v2, extracted or raw representation");
        if ((c.observation & kObsSmm) &&
            (c.smmWidth < 1 || c.smmHeight < 1 || c.smmWidth > 4096 || c.smmHeight > 4096))
            throw std::invalid_argument("expected SMM dimensions from 1 to 4096, found " + std::to_string(c.smmWidth) +
                                        " x " + std::to_string(c.smmHeight));
        if (c.assets.empty()) throw std::invalid_argument("expected an asset bundle");
        if (c.ticksPerStep < 1)
            throw std::invalid_argument("expected at least one tick in a step, found " + std::to_string(c.ticksPerStep));
        if (!c.fixedSeeds.empty()) {
            if ((int)c.fixedSeeds.size() != c.count)
                throw std::invalid_argument("expected one fixed seed for each environment, found " +
                                            std::to_string(c.fixedSeeds.size()));
            for (int64_t s : c.fixedSeeds)
                if (s < -1 || s > 4294967295LL)
                    throw std::invalid_argument("expected a fixed seed from 0 to 4294967295, found " + std::to_string(s));
        }
        if (c.firstIndex < 0 || c.firstIndex + c.count > (int64_t(1) << 32))
            throw std::invalid_argument("expected a first index from 0 to 2**32 minus the environment count, found " +
                                        std::to_string(c.firstIndex));
        if (c.episodeNumber < 0)
            throw std::invalid_argument("expected an episode number of at least 0, found " + std::to_string(c.episodeNumber));
        if (c.stack != 1 && c.stack != 4)
            throw std::invalid_argument("expected a stack of 1 or 4 observations, found " + std::to_string(c.stack));
        if (c.actionSet < 0 || c.actionSet > 2) throw std::invalid_argument("expected an action set from 0 to 2");
        std::vector<int32_t> assignment = c.assignment;
        if (assignment.empty()) assignment.assign(c.count, 0);
        if ((int)assignment.size() != c.count)
            throw std::invalid_argument("expected one bundle for each of the " + std::to_string(c.count) +
                                        " environments, found " + std::to_string(assignment.size()));
        for (int32_t x : assignment)
            if (x < 0 || x >= (int)c.assets.size())
                throw std::invalid_argument("expected a bundle from 0 to " + std::to_string(c.assets.size() - 1) +
                                            ", found " + std::to_string(x));
        if (!c.agentCounts.empty() && c.agentCounts.size() != 2 * c.assets.size())
            throw std::invalid_argument("expected a left and a right agent count for each bundle");
        for (size_t i = 0; i < c.assets.size(); i++) {
            const int l = c.agentCounts.empty() ? -1 : c.agentCounts[2 * i];
            const int r = c.agentCounts.empty() ? -1 : c.agentCounts[2 * i + 1];
            bundles.push_back(load_assets(c.assets[i], l, r));
        }
        store = parse_animations(read_file(c.animations));

        // Shared tables.
        const AnimStore &st = *store;
        AnimTables t{};
        t.anims = upload(st.anims);
        t.derived = upload(st.derived);
        t.nodes = upload(st.nodes);
        t.keys = upload(st.keys);
        t.interp = upload(st.interp);
        t.football = upload(st.football);
        t.positions = upload(st.positions);
        t.quadrants = upload(st.quadrants);
        t.functionAnims = upload(st.functionAnims);
        t.functionOffsets = upload(st.functionOffsets);
        t.smoothed = upload(st.smoothed);
        t.animCount = (int32_t)st.anims.size();
        t.quadrantCount = (int32_t)st.quadrants.size();
        t.maxIncomingBallDirDeviation = st.maxIn;
        t.maxOutgoingBallDirDeviation = st.maxOut;
        const AnimTables *tDev = upload(&t, 1);
        const float *camDev = upload(st.cameraWeights);

        // Variants: bundle * 4 + reverse * 2 + parity.
        int agents = 0;
        for (const Assets &bd : bundles) {
            if (bd.leftAgents < 0 || bd.rightAgents < 0 || bd.leftAgents + bd.rightAgents > kAgentsMax)
                throw std::runtime_error("expected at most 22 agents in a bundle");
            agents = std::max(agents, bd.leftAgents + bd.rightAgents);
            for (const AssetVariant &v : bd.variants) {
                const Scenario &sc = v.world->scenario;
                players = std::max({players, (int)sc.leftTeamSize, (int)sc.rightTeamSize});
                if (sc.controlAllPlayers && dynamic_player_selection(*v.world))
                    throw std::invalid_argument(
                        "expected 0 or all the controllable players of a side as agents for a scenario with "
                        "control_all_players");
                const int64_t seconds = (int64_t)sc.gameDuration * c.ticksPerStep / 100 + 1;
                if (seconds > 512)
                    throw std::invalid_argument("expected a match of at most 512 seconds of play, the position history "
                                                "of a player");
                Variant hv{};
                hv.tmpl = upload(v.world.get(), 1);
                hv.ctx.anim = tDev;
                hv.ctx.staticData = upload(&v.staticData, 1);
                hv.ctx.skeletons = upload(v.skeletons);
                hv.ctx.cameraWeights = camDev;
                hv.ctx.ticksPerStep = c.ticksPerStep;
                hostVariants.push_back(hv);
            }
        }
        b.variants = upload(hostVariants);
        b.count = c.count;
        b.agents = agents;
        b.actionSet = c.actionSet;
        b.observation = c.observation;
        b.checkpoints = c.checkpoints;
        b.numpyLegacy = c.numpyLegacy;
        b.autoReset = c.autoReset;
        b.stack = c.stack;
        b.worlds = alloc<Match>(c.count);
        b.cores = alloc<EnvCore>(c.count);
        b.slots = alloc<EnvSlot>(c.count);
        b.scratch = alloc<WarpScratch>(c.count);
        if (!estimate) check(default_crew_log2(c.count, &b.crewLog2), "launch geometry");
        b.status = alloc<int32_t>(c.count);
        b.anyFail = alloc<int32_t>(1);
        b.reward = alloc<float>((size_t)c.count * agents);
        b.done = alloc<uint8_t>(c.count);
        b.scoreReward = alloc<int32_t>(c.count);
        if (c.observation & (kObsSimple115 | kObsSimple115v2)) {
            b.simple115 = alloc<float>((size_t)c.count * agents * kSimple115 * c.stack);
            b.finalSimple115 = alloc<float>((size_t)c.count * agents * kSimple115 * c.stack);
        }
        b.smmWidth = c.smmWidth;
        b.smmHeight = c.smmHeight;
        if (c.observation & kObsRaw) {
            b.rawLayout = make_raw_layout((size_t)c.count * agents, players, sticky_count(c.actionSet));
            b.raw = alloc<uint8_t>(b.rawLayout.bytes);
            b.finalRaw = alloc<uint8_t>(b.rawLayout.bytes);
        }
        if (c.observation & kObsSmm) {
            // Zero maps and no marks: the first write paints onto a clear map.
            const size_t map = (size_t)c.smmWidth * c.smmHeight * kSmmLayers * c.stack;
            const size_t marks = (size_t)kSmmMarkRow * c.stack;
            b.smm = alloc<uint8_t>((size_t)c.count * agents * map);
            b.finalSmm = alloc<uint8_t>((size_t)c.count * agents * map);
            b.smmMarks = alloc<int32_t>((size_t)c.count * agents * marks);
            b.finalSmmMarks = alloc<int32_t>((size_t)c.count * agents * marks);
        }
        b.teamDifficulty = nullptr;
        actionsDev = alloc<int32_t>((size_t)c.count * agents);
        maskDev = alloc<uint8_t>(c.count);
        seedsDev = alloc<int64_t>(c.count);
        reverseDev = alloc<int32_t>(c.count);
        outputMaskDev = alloc<uint8_t>(c.count);
        hostSlots.resize(c.count);
        for (int e = 0; e < c.count; e++) {
            EnvSlot &s = hostSlots[e];
            memset(&s, 0, sizeof(s));
            episode_seed(s.gen, c.seed, (uint32_t)(c.firstIndex + e));
            s.fixedSeed = c.fixedSeeds.empty() ? -1 : c.fixedSeeds[e];
            s.episodeOffset = c.episodeNumber;
            s.bundle = assignment[e];
            s.leftAgents = bundles[s.bundle].leftAgents;
            s.rightAgents = bundles[s.bundle].rightAgents;
        }
        if (!estimate) check(cudaMemcpy(b.slots, hostSlots.data(), sizeof(EnvSlot) * c.count, cudaMemcpyHostToDevice), "slots");
        if (!estimate) reserve_stack();
        started.assign(c.count, false);
        unstarted = c.count;
    }

    // The kernels' call chains are deep (AI, selection, physics): the per-thread stack is set to
    // twice what the compiler reports for the deepest kernel, so no call chain can outgrow it.
    void reserve_stack() {
        size_t local = 0;
        int regs = 0;
        check(kernel_attributes(&local, &regs), "kernel attributes");
        size_t current = 0;
        check(cudaDeviceGetLimit(&current, cudaLimitStackSize), "stack limit");
        const size_t want = (2 * local + 1023) & ~(size_t)1023;
        if (current < want) check(cudaDeviceSetLimit(cudaLimitStackSize, want), "stack limit");
    }

    const AssetVariant &variant(int v) const { return bundles[v / 4].variants[v % 4]; }
    const Scenario &scenario(int e) const { return variant(hostSlots[e].bundle * 4).world->scenario; }

    // Waits for `stream` and turns a failed environment into an error.
    void sync(cudaStream_t stream) {
        check(cudaStreamSynchronize(stream), "the batch's device work");
        int32_t f = 0;
        check(cudaMemcpy(&f, b.anyFail, 4, cudaMemcpyDeviceToHost), "status");
        if (f == kStatusUnsupported)
            throw std::runtime_error("an environment reached a path that GRF leaves undefined");
        if (f == kStatusOverflow) throw std::runtime_error("an environment outgrew a fixed capacity of its state");
        if (f) throw std::runtime_error("an environment failed with code " + std::to_string(f));
    }
    void check_reverse(const int32_t *r) const {
        for (int e = 0; e < b.count; e++)
            if (r[e] != 0 && r[e] != 1)
                throw std::invalid_argument("the reverse flag of environment " + std::to_string(e) + " is " +
                                            std::to_string(r[e]) + ", not 0 or 1");
    }
    void check_seeds(const int64_t *s) const {
        for (int e = 0; e < b.count; e++)
            if (s[e] < -1 || s[e] > 4294967295LL)
                throw std::invalid_argument("expected seeds from 0 to 4294967295, or -1 to draw, found " +
                                            std::to_string(s[e]) + " for environment " + std::to_string(e));
    }
    void check_started() const {
        if (unstarted > 0)
            throw std::logic_error("expected a reset of the batch, or a state for every environment, before its first step");
    }
    void check_actions(const int32_t *a) const {
        const int n = action_set_size(b.actionSet);
        for (int e = 0; e < b.count; e++) {
            const EnvSlot &s = hostSlots[e];
            const int32_t *row = a + (size_t)e * b.agents;
            for (int k = 0; k < s.leftAgents + s.rightAgents; k++)
                if (row[k] < -n || row[k] >= n)
                    throw std::out_of_range("expected action indices from " + std::to_string(-n) + " to " +
                                            std::to_string(n - 1) + ", found " + std::to_string(row[k]));
        }
    }
    void check_env(int e) const {
        if (e < 0 || e >= b.count)
            throw std::invalid_argument("expected an environment from 0 to " + std::to_string(b.count - 1) +
                                        ", found " + std::to_string(e));
    }

    void reset(const uint32_t *seeds, const int32_t *reverse, cudaStream_t stream) {
        const int64_t *sd = nullptr;
        const int32_t *rd = nullptr;
        if (seeds) {
            std::vector<int64_t> wide(seeds, seeds + b.count);
            check(cudaMemcpyAsync(seedsDev, wide.data(), 8 * (size_t)b.count, cudaMemcpyHostToDevice, stream), "seeds");
            check(cudaStreamSynchronize(stream), "seeds");
            sd = seedsDev;
        }
        if (reverse) {
            check_reverse(reverse);
            check(cudaMemcpyAsync(reverseDev, reverse, 4 * (size_t)b.count, cudaMemcpyHostToDevice, stream), "reverse");
            rd = reverseDev;
        }
        check(launch_reset(b, nullptr, sd, rd, stream), "reset launch");
        sync(stream);
        started.assign(b.count, true);
        unstarted = 0;
    }
    void reset_masked(const uint8_t *mask, bool onDevice, const int64_t *seeds, const int32_t *reverse,
                      cudaStream_t stream) {
        const int n = b.count;
        if (seeds) check_seeds(seeds);
        if (reverse) check_reverse(reverse);
        const uint8_t *md = mask;
        if (mask && !onDevice) {
            check(cudaMemcpyAsync(maskDev, mask, (size_t)n, cudaMemcpyHostToDevice, stream), "mask");
            md = maskDev;
        }
        const int64_t *sd = nullptr;
        if (seeds) {
            check(cudaMemcpyAsync(seedsDev, seeds, 8 * (size_t)n, cudaMemcpyHostToDevice, stream), "seeds");
            sd = seedsDev;
        }
        const int32_t *rd = nullptr;
        if (reverse) {
            check(cudaMemcpyAsync(reverseDev, reverse, 4 * (size_t)n, cudaMemcpyHostToDevice, stream), "reverse");
            rd = reverseDev;
        }
        if (unstarted > 0) {
            std::vector<uint8_t> st(n, 1);
            if (mask && onDevice) {
                check(cudaStreamSynchronize(stream), "mask");
                check(cudaMemcpy(st.data(), mask, (size_t)n, cudaMemcpyDeviceToHost), "mask");
            } else if (mask) {
                st.assign(mask, mask + n);
            }
            for (int e = 0; e < n; e++)
                if (st[e] && !started[e]) {
                    started[e] = true;
                    unstarted--;
                }
        }
        check(launch_reset(b, md, sd, rd, stream), "reset launch");
        if (mask && !onDevice) check(cudaStreamSynchronize(stream), "host mask");
    }
    // Masked reset with the mask and seeds already in device memory: nothing is read back or
    // checked on the host and nothing synchronises, so the call can sit in a captured graph beside
    // the step. The started books need the mask on the host, so a device mask is refused until
    // every environment has started (a reset without a mask starts them all).
    void reset_masked_device(const uint8_t *mask, const int64_t *seeds, cudaStream_t stream) {
        if (mask && unstarted > 0)
            throw std::logic_error("expected every environment started (a reset of the whole batch) before a "
                                   "masked reset with a device mask");
        check(launch_reset(b, mask, seeds, nullptr, stream), "reset launch");
        if (!mask && unstarted > 0) {
            started.assign(b.count, true);
            unstarted = 0;
        }
    }
    void step(const int32_t *actions, bool onDevice, cudaStream_t stream, bool synchronize) {
        check_started();
        const int32_t *ad = actions;
        if (!onDevice) {
            check_actions(actions);
            check(cudaMemcpyAsync(actionsDev, actions, 4 * (size_t)b.count * b.agents, cudaMemcpyHostToDevice, stream),
                  "actions");
            ad = actionsDev;
        }
        check(launch_step(b, ad, stream), "step launch");
        if (synchronize) sync(stream);
        else if (!onDevice) check(cudaStreamSynchronize(stream), "host actions");
    }
    // The step with device-resident actions and the fixed sort scratch of kernels.cu in place of
    // the batch's own: no allocation of any kind. Returns null, or the reason for refusing.
    const char *step_static(const int32_t *actions, cudaStream_t stream, char *message, size_t size) {
        if (unstarted > 0) return "expected a reset of the batch before its first step";
        if (b.count > kStaticScratchEnvironments) {
            snprintf(message, size, "expected at most %d environments for the static-scratch step, found %d",
                     kStaticScratchEnvironments, b.count);
            return message;
        }
        if (!actions) return "expected device actions";
        int device = -1;
        if (cudaGetDevice(&device) != cudaSuccess) return "no current CUDA device";
        // A failed attribute query leaves a non-sticky error behind. It is cleared so that a later
        // launch check does not report it, but only when no error was pending before this call: an
        // error the caller has not read yet stays for the caller.
        const bool errorPending = cudaPeekAtLastError() != cudaSuccess;
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, actions) != cudaSuccess) {
            if (!errorPending) (void)cudaGetLastError();
            return "expected actions in device memory of the current device";
        }
        if ((a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) || a.device != device)
            return "expected actions in device memory of the current device";
        cudaPointerAttributes own{};
        if (cudaPointerGetAttributes(&own, b.status) != cudaSuccess) {
            if (!errorPending) (void)cudaGetLastError();
            return "expected the batch's device to be the current device";
        }
        if (own.device != device) return "expected the batch's device to be the current device";
        WarpScratch *scratch = nullptr;
        cudaError_t rc = static_scratch_address(&scratch);
        if (rc == cudaSuccess) {
            Batch view = b;
            view.scratch = scratch;
            rc = launch_step(view, actions, stream);
        }
        if (rc != cudaSuccess) {
            snprintf(message, size, "static-scratch step: %s", cudaGetErrorString(rc));
            return message;
        }
        return nullptr;
    }
    void reset_done(cudaStream_t stream) {
        check_started();
        check(launch_reset(b, b.done, nullptr, nullptr, stream), "reset launch");
    }
    void set_difficulty(const float *d) {
        const size_t n = (size_t)b.count * 2;
        for (size_t i = 0; i < n; i++)
            if (!(d[i] <= 1)) throw std::invalid_argument("expected a difficulty from 0 to 1, found " + std::to_string(d[i]));
        if (!b.teamDifficulty) b.teamDifficulty = alloc<float>(n);
        check(cudaMemcpy(const_cast<float *>(b.teamDifficulty), d, n * 4, cudaMemcpyHostToDevice), "difficulty");
        hostDifficulty.assign(d, d + n);
    }
    float difficulty(int e, int side) const {
        if (!hostDifficulty.empty() && hostDifficulty[e * 2 + side] >= 0.0f) return hostDifficulty[e * 2 + side];
        const Scenario &sc = variant(hostSlots[e].bundle * 4 + (cfg.episodeNumber & 1)).world->scenario;
        return side == 0 ? sc.leftTeamDifficulty : sc.rightTeamDifficulty;
    }
    // batch_environment.h:396 (SetState). The state's scenario picks the variant (of the
    // environment's bundle) to continue from; its difficulties must be the environment's. The
    // observation is computed on the host from the loaded world, reward, done and score restart at
    // zero, and the outputs are written as after a reset.
    void set_state(int e, const std::string &bytes, int prevScoreDiff, int prevGameMode, int prevBallOwnedTeam,
                   const int32_t *collected) {
        check_env(e);
        check(cudaDeviceSynchronize(), "set_state");
        std::unique_ptr<Match> w(new Match);
        Codec codec;
        codec.animationCount = (int)store->anims.size();
        if (!codec.load_frame(bytes, *w))
            throw std::invalid_argument("expected the bytes of a state, found bytes that do not load");
        const int bundle = hostSlots[e].bundle;
        // The scenario compares without the state's real_time flag; the bundle's stands in.
        const bool realTime = w->scenario.realTime;
        w->scenario.realTime = bundles[bundle].variants[0].world->scenario.realTime;
        const std::string sc = save_scenario(*w);
        int parity = 0;
        while (parity < 4 && bundles[bundle].variants[parity].scenario != sc) parity++;
        if (parity == 4) throw std::invalid_argument("expected a state of the scenario of the environment, found another");
        w->scenario.realTime = realTime;
        const Scenario &own = bundles[bundle].variants[parity].world->scenario;
        float expected[2] = {own.leftTeamDifficulty, own.rightTeamDifficulty};
        for (int side = 0; side < 2; side++)
            if (!hostDifficulty.empty() && hostDifficulty[e * 2 + side] >= 0.0f) expected[side] = hostDifficulty[e * 2 + side];
        if (memcmp(&w->scenario.leftTeamDifficulty, &expected[0], 4) != 0 ||
            memcmp(&w->scenario.rightTeamDifficulty, &expected[1], 4) != 0)
            throw std::invalid_argument("expected a state of the difficulties of the environment, " +
                                        std::to_string(expected[0]) + " and " + std::to_string(expected[1]) +
                                        ", found " + std::to_string(w->scenario.leftTeamDifficulty) + " and " +
                                        std::to_string(w->scenario.rightTeamDifficulty));
        const int variantIndex = bundle * 4 + parity;
        const AssetVariant &av = bundles[bundle].variants[parity];
        std::unique_ptr<EnvCore> core(new EnvCore{});
        core->previousScoreDifference = prevScoreDiff;
        core->previousGameMode = prevGameMode;
        core->previousBallOwnedTeam = prevBallOwnedTeam;
        Context ctx{};
        ctx.staticData = &av.staticData;
        ctx.skeletons = av.skeletons.data();
        ctx.ticksPerStep = cfg.ticksPerStep;
        environment_get_state(*w, ctx, core->observation);
        EnvSlot slot;
        check(cudaMemcpy(&slot, b.slots + e, sizeof(EnvSlot), cudaMemcpyDeviceToHost), "set_state");
        slot.variant = variantIndex;
        const int agents = slot.leftAgents + slot.rightAgents;
        for (int a = 0; a < kAgentsMax; a++) slot.collected[a] = collected && a < agents ? collected[a] : 0;
        for (int a = 0; a < agents; a++) {
            const bool left = a < slot.leftAgents;
            for (int i = 0; i < sticky_count(b.actionSet); i++)
                slot.sticky[a][i] = sticky_action_state(*w, sticky_action(i), left, left ? a : a - slot.leftAgents);
        }
        // A sent-off keeper's hand-over lives outside the state, so it carries over.
        check(cudaMemcpy(w->formationOverride, b.worlds[e].formationOverride, sizeof(w->formationOverride),
                         cudaMemcpyDeviceToHost),
              "set_state");
        check(cudaMemcpy(b.worlds + e, w.get(), sizeof(Match), cudaMemcpyHostToDevice), "set_state");
        check(cudaMemcpy(b.cores + e, core.get(), sizeof(EnvCore), cudaMemcpyHostToDevice), "set_state");
        check(cudaMemcpy(b.slots + e, &slot, sizeof(EnvSlot), cudaMemcpyHostToDevice), "set_state");
        check(cudaMemset(b.reward + (size_t)e * b.agents, 0, sizeof(float) * b.agents), "set_state");
        check(cudaMemset(b.done + e, 0, 1), "set_state");
        check(cudaMemset(b.scoreReward + e, 0, sizeof(int32_t)), "set_state");
        check(cudaMemset(b.status + e, 0, sizeof(int32_t)), "set_state");
        check(cudaMemset(outputMaskDev, 0, (size_t)b.count), "set_state");
        check(cudaMemset(outputMaskDev + e, 1, 1), "set_state");
        check(launch_outputs(b, outputMaskDev, nullptr), "set_state outputs");
        check(cudaDeviceSynchronize(), "set_state");
        if (!started[e]) {
            started[e] = true;
            unstarted--;
        }
    }
    // stacked_state.h:23 (SetStackedFrames): the observation stack of environment `e` after
    // set_state, the oldest frame first: `[agents][115 * stack]` float32 for simple115, or
    // `[agents][height][width][4 * stack]` uint8 for smm, whose frames must hold only 0 and 255
    // (at most kSmmMarks cells of 255 a frame); their marks are rebuilt so that the next step
    // clears exactly the marked bytes.
    void set_stack(int e, const std::string &name, const void *frames, size_t size) {
        check_env(e);
        if (b.stack < 2) throw std::invalid_argument("expected a batch that stacks its observations");
        if (name == "smm" && b.smm) {
            set_smm_stack(e, static_cast<const uint8_t *>(frames), size);
            return;
        }
        if (name != "simple115" || !b.simple115)
            throw std::invalid_argument("expected the stack simple115 or smm of the batch, found " + name);
        const size_t agents = (size_t)(hostSlots[e].leftAgents + hostSlots[e].rightAgents);
        const size_t width = (size_t)kSimple115 * b.stack;
        const size_t expected = agents * width * sizeof(float);
        if (size != expected)
            throw std::invalid_argument("expected a stack of " + std::to_string(expected) +
                                        " bytes for the agents of environment " + std::to_string(e) + ", found " +
                                        std::to_string(size));
        check(cudaDeviceSynchronize(), "set_stack");
        check(cudaMemcpy(b.simple115 + (size_t)e * b.agents * width, frames, size, cudaMemcpyHostToDevice), "set_stack");
    }
    void set_smm_stack(int e, const uint8_t *bytes, size_t size) {
        const size_t agents = (size_t)(hostSlots[e].leftAgents + hostSlots[e].rightAgents);
        const int stack = b.stack;
        const size_t frameBytes = (size_t)b.smmWidth * b.smmHeight * kSmmLayers;
        const size_t agentBytes = frameBytes * stack;
        if (size != agents * agentBytes)
            throw std::invalid_argument("expected a stack of " + std::to_string(agents * agentBytes) +
                                        " bytes for the agents of environment " + std::to_string(e) + ", found " +
                                        std::to_string(size));
        std::vector<int32_t> marks(agents * stack * kSmmMarkRow, 0);
        for (size_t a = 0; a < agents; a++)
            for (int f = 0; f < stack; f++) {
                int32_t *row = marks.data() + (a * stack + f) * kSmmMarkRow;
                for (size_t m = 0; m < frameBytes; m++) {
                    const uint8_t v = bytes[a * agentBytes + m / kSmmLayers * kSmmLayers * stack + kSmmLayers * f +
                                            m % kSmmLayers];
                    if (v == 0) continue;
                    if (v != 255 || row[0] == kSmmMarks)
                        throw std::invalid_argument("expected a minimap of GRF, of at most " + std::to_string(kSmmMarks) +
                                                    " cells of 255 a frame and zeros, found a cell of " +
                                                    std::to_string(v));
                    row[1 + row[0]++] = (int32_t)m;
                }
            }
        check(cudaDeviceSynchronize(), "set_stack");
        const size_t first = (size_t)e * b.agents;
        check(cudaMemcpy(b.smm + first * agentBytes, bytes, size, cudaMemcpyHostToDevice), "set_stack");
        check(cudaMemcpy(b.smmMarks + first * kSmmMarkRow * stack, marks.data(), marks.size() * sizeof(int32_t),
                         cudaMemcpyHostToDevice),
              "set_stack");
    }
    std::string get_state(int e, EnvCore &core, EnvSlot &slot) {
        check_env(e);
        check(cudaDeviceSynchronize(), "get_state");
        std::unique_ptr<Match> w(new Match);
        check(cudaMemcpy(w.get(), b.worlds + e, sizeof(Match), cudaMemcpyDeviceToHost), "get_state");
        check(cudaMemcpy(&core, b.cores + e, sizeof(EnvCore), cudaMemcpyDeviceToHost), "get_state");
        check(cudaMemcpy(&slot, b.slots + e, sizeof(EnvSlot), cudaMemcpyDeviceToHost), "get_state");
        Codec codec;
        codec.freeControllerCount = variant(slot.variant).freeControllerCount;
        return codec.save_frame(*w);
    }
};

}  // namespace host
}  // namespace cb

using cb::host::BatchEnv;

namespace {
thread_local std::string lastError;
thread_local unsigned long long *memoryEstimate = nullptr;
int fail(const std::exception &e) {
    lastError = e.what();
    return -1;
}
cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }
}  // namespace

#pragma GCC visibility push(default)
extern "C" {

const char *cuju_last_error() { return lastError.c_str(); }
const char *cuju_backend() { return "cuda"; }

void *cuju_environment_create(const cuju_configuration *s) {
    try {
        lastError.clear();
        if (s->version != CUJU_CONFIGURATION_VERSION)
            throw std::invalid_argument("expected the configuration version 2, found " + std::to_string(s->version));
        if (s->environment_count < 1)
            throw std::invalid_argument("expected at least one environment, found " + std::to_string(s->environment_count));
        cb::host::Config c;
        c.assets.assign(s->assets, s->assets + s->asset_count);
        if (s->assignment) c.assignment.assign(s->assignment, s->assignment + s->environment_count);
        c.animations = s->animations;
        c.count = s->environment_count;
        c.seed = s->seed;
        c.actionSet = s->action_set;
        c.observation = s->observation;
        c.checkpoints = s->checkpoints != 0;
        c.numpyLegacy = s->numpy_legacy != 0;
        c.autoReset = s->auto_reset != 0;
        c.ticksPerStep = s->ticks_per_step;
        c.smmWidth = s->smm_width;
        c.smmHeight = s->smm_height;
        c.stack = s->stack;
        if (s->fixed_seeds) c.fixedSeeds.assign(s->fixed_seeds, s->fixed_seeds + s->environment_count);
        if (s->agent_counts) c.agentCounts.assign(s->agent_counts, s->agent_counts + 2 * s->asset_count);
        c.episodeNumber = s->episode_number;
        c.firstIndex = (int64_t)std::min(s->first_index, 1ULL << 62);
        c.allocate = s->allocate;
        c.release = s->release;
        c.allocatorContext = s->allocator_context;
        std::unique_ptr<BatchEnv> env(new BatchEnv(c, memoryEstimate));
        // An estimate only counts the bytes; no batch comes out of it.
        if (memoryEstimate) return nullptr;
        return env.release();
    } catch (const std::exception &e) {
        fail(e);
        return nullptr;
    }
}

int cuju_memory_estimate(const cuju_configuration *s, unsigned long long *bytes) {
    *bytes = 0;
    memoryEstimate = bytes;
    cuju_environment_create(s);
    memoryEstimate = nullptr;
    return lastError.empty() ? 0 : -1;
}

int cuju_local_memory_bytes(unsigned long long *bytes) {
    try {
        size_t local = 0;
        int regs = 0;
        cb::host::check(cb::kernel_attributes(&local, &regs), "kernel attributes");
        int dev = 0, sms = 0, threads = 0;
        cb::host::check(cudaGetDevice(&dev), "device");
        cb::host::check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "device");
        cb::host::check(cudaDeviceGetAttribute(&threads, cudaDevAttrMaxThreadsPerMultiProcessor, dev), "device");
        *bytes = (unsigned long long)local * sms * threads;
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}

unsigned long long cuju_environment_memory_bytes(void *env) { return static_cast<BatchEnv *>(env)->mem.bytes; }
void cuju_environment_destroy(void *env) { delete static_cast<BatchEnv *>(env); }
int cuju_environment_count(void *env) { return static_cast<BatchEnv *>(env)->b.count; }
int cuju_environment_threads(void *) { return 0; }

int cuju_environment_agents(void *env, int *left, int *right) {
    const BatchEnv *e = static_cast<BatchEnv *>(env);
    for (int i = 0; i < e->b.count; i++) {
        if (left) left[i] = e->hostSlots[i].leftAgents;
        if (right) right[i] = e->hostSlots[i].rightAgents;
    }
    return e->b.agents;
}
int cuju_environment_players(void *env, int *left, int *right) {
    const BatchEnv *e = static_cast<BatchEnv *>(env);
    for (int i = 0; i < e->b.count; i++) {
        if (left) left[i] = e->scenario(i).leftTeamSize;
        if (right) right[i] = e->scenario(i).rightTeamSize;
    }
    return e->players;
}
int cuju_environment_set_difficulty(void *env, const float *difficulty) {
    try {
        static_cast<BatchEnv *>(env)->set_difficulty(difficulty);
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
void cuju_environment_difficulty(void *env, float *difficulty) {
    const BatchEnv *e = static_cast<BatchEnv *>(env);
    for (int i = 0; i < e->b.count; i++)
        for (int s = 0; s < 2; s++) difficulty[i * 2 + s] = e->difficulty(i, s);
}
int cuju_environment_reset(void *env, const unsigned int *seeds, const int *reverse, void *stream) {
    try {
        static_cast<BatchEnv *>(env)->reset(seeds, reverse, as_stream(stream));
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
int cuju_environment_reset_masked(void *env, const unsigned char *mask, int mask_on_device, const int64_t *seeds,
                                  const int *reverse, void *stream, int synchronize) {
    try {
        BatchEnv *e = static_cast<BatchEnv *>(env);
        e->reset_masked(mask, mask_on_device != 0, seeds, reverse, as_stream(stream));
        if (synchronize) e->sync(as_stream(stream));
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
// No reference counterpart: see include/cuju_b200.h.
int cuju_b200_environment_reset_masked_device(void *env, const unsigned char *mask, const long long *seeds,
                                              void *stream) {
    try {
        static_cast<BatchEnv *>(env)->reset_masked_device(mask, reinterpret_cast<const int64_t *>(seeds),
                                                          as_stream(stream));
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
int cuju_b200_environment_set_lanes(void *env, int lanes) {
    try {
        BatchEnv &batch = *static_cast<BatchEnv *>(env);
        int log2 = -1;
        for (int k = 0; k <= 5; k++)
            if (lanes == (1 << k)) log2 = k;
        if (lanes == 0) cb::host::check(cb::default_crew_log2(batch.b.count, &log2), "launch geometry");
        if (log2 < 0)
            throw std::invalid_argument("expected 0 (the default) or 1, 2, 4, 8, 16 or 32 lanes per environment, found " +
                                        std::to_string(lanes));
        batch.b.crewLog2 = log2;
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
int cuju_environment_reset_done(void *env, void *stream) {
    try {
        static_cast<BatchEnv *>(env)->reset_done(as_stream(stream));
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
int cuju_environment_step(void *env, const int *actions, int on_device, void *stream, int synchronize) {
    try {
        static_cast<BatchEnv *>(env)->step(actions, on_device != 0, as_stream(stream), synchronize != 0);
        return 0;
    } catch (const std::out_of_range &e) {
        fail(e);
        return -2;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
// No reference counterpart: see include/cuju_b200.h. The success path allocates nothing.
int cuju_b200_environment_step_static(void *env, const int *actions, void *stream) {
    thread_local char message[160];
    const char *why = static_cast<BatchEnv *>(env)->step_static(actions, as_stream(stream), message, sizeof message);
    if (!why) return 0;
    lastError.assign(why);
    return -1;
}
int cuju_environment_step_async(void *env, const int *actions, int on_device, void *stream) {
    try {
        static_cast<BatchEnv *>(env)->step(actions, on_device != 0, as_stream(stream), false);
        return 0;
    } catch (const std::out_of_range &e) {
        fail(e);
        return -2;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
int cuju_environment_step_wait(void *) { return 0; }
int cuju_environment_synchronize(void *env, void *stream) {
    try {
        static_cast<BatchEnv *>(env)->sync(as_stream(stream));
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
const char *cuju_environment_get_state(void *env, int index, unsigned long long *size, int *episode) {
    thread_local std::string bytes;
    try {
        BatchEnv *e = static_cast<BatchEnv *>(env);
        std::unique_ptr<cb::EnvCore> core(new cb::EnvCore);
        cb::EnvSlot slot;
        bytes = e->get_state(index, *core, slot);
        *size = bytes.size();
        episode[0] = core->previousScoreDifference;
        episode[1] = core->previousGameMode;
        episode[2] = core->previousBallOwnedTeam;
        for (int a = 0; a < e->b.agents; a++) episode[3 + a] = slot.collected[a];
        return bytes.data();
    } catch (const std::exception &ex) {
        fail(ex);
        return nullptr;
    }
}
int cuju_environment_set_state(void *env, int index, const char *bytes, unsigned long long size, const int *episode) {
    try {
        if (!bytes || !episode) throw std::invalid_argument("expected state bytes and episode values");
        static_cast<BatchEnv *>(env)->set_state(index, std::string(bytes, size), episode[0], episode[1], episode[2],
                                                episode + 3);
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
int cuju_environment_set_stack(void *env, int index, const char *name, const void *frames, unsigned long long size) {
    try {
        if (!name || !frames) throw std::invalid_argument("expected a stack name and its frames");
        static_cast<BatchEnv *>(env)->set_stack(index, name, frames, size);
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
void *cuju_environment_buffer(void *env, const char *name) {
    const cb::Batch &b = static_cast<BatchEnv *>(env)->b;
    const std::string n = name;
    if (n == "simple115") return b.simple115;
    if (n == "final_simple115") return b.finalSimple115;
    if (n == "smm") return b.smm;
    if (n == "final_smm") return b.finalSmm;
    if (n == "raw") return b.raw;
    if (n == "final_raw") return b.finalRaw;
    if (n == "reward") return b.reward;
    if (n == "done") return b.done;
    if (n == "score_reward") return b.scoreReward;
    return nullptr;
}
const char *cuju_environment_raw_field(void *env, int field, int *type, int *dimensions, unsigned long long *offset) {
    static const char *const names[cb::kRawFields] = {
        "ball", "ball_direction", "ball_rotation", "ball_owned_team", "ball_owned_player", "left_team",
        "left_team_direction", "left_team_tired_factor", "left_team_yellow_card", "left_team_active",
        "left_team_roles", "right_team", "right_team_direction", "right_team_tired_factor",
        "right_team_yellow_card", "right_team_active", "right_team_roles", "score", "steps_left", "game_mode",
        "active", "designated", "sticky_actions"};
    const cb::Batch &b = static_cast<BatchEnv *>(env)->b;
    if (!b.raw || field < 0 || field >= cb::kRawFields) return nullptr;
    const cb::RawArray &a = b.rawLayout.arrays[field];
    *type = a.type;
    dimensions[0] = a.dims[0];
    dimensions[1] = a.dims[1];
    *offset = a.offset;
    return names[field];
}
int cuju_environment_episode(void *env, int index, long long *values, float *difficulty) {
    try {
        BatchEnv *e = static_cast<BatchEnv *>(env);
        e->check_env(index);
        cb::EnvSlot slot;
        cb::host::check(cudaMemcpy(&slot, e->b.slots + index, sizeof(slot), cudaMemcpyDeviceToHost), "episode");
        std::unique_ptr<cb::Observation> o(new cb::Observation);
        cb::host::check(cudaMemcpy(o.get(), &e->b.cores[index].observation, sizeof(cb::Observation), cudaMemcpyDeviceToHost),
                        "episode");
        const cb::host::Assets &bd = e->bundles[slot.bundle];
        const cb::Scenario &sc = bd.variants[0].world->scenario;
        values[0] = slot.seed;
        values[1] = slot.reverse;
        values[2] = slot.episode;
        values[3] = slot.episodeOffset;
        values[4] = slot.bundle;
        values[5] = o->step;
        values[6] = slot.fixedSeed;
        values[7] = sc.deterministic;
        values[8] = e->cfg.ticksPerStep;
        values[9] = slot.leftAgents;
        values[10] = slot.rightAgents;
        values[11] = sc.leftTeamSize;
        values[12] = sc.rightTeamSize;
        for (int t = 0; t < 2; t++) {
            values[13 + t] = o->team[t].designatedPlayer;
            values[15 + t] = slot.finalDesignated[t];
        }
        if (difficulty) {
            const cb::Scenario &played = e->b.worlds[index].scenario;
            cb::host::check(cudaMemcpy(&difficulty[0], &played.leftTeamDifficulty, 4, cudaMemcpyDeviceToHost), "episode");
            cb::host::check(cudaMemcpy(&difficulty[1], &played.rightTeamDifficulty, 4, cudaMemcpyDeviceToHost), "episode");
            const cb::Scenario &own = bd.variants[slot.variant % 4].world->scenario;
            difficulty[2] = own.leftTeamDifficulty;
            difficulty[3] = own.rightTeamDifficulty;
        }
        return 0;
    } catch (const std::exception &ex) {
        return fail(ex);
    }
}
const char *cuju_environment_scenario(void *env, int bundle) {
    const BatchEnv *e = static_cast<BatchEnv *>(env);
    if (bundle < 0 || bundle >= (int)e->bundles.size()) return nullptr;
    return e->bundles[bundle].scenario.c_str();
}
// No reference counterpart: the kernels' per-thread local memory and registers and the current
// per-thread stack limit, for diagnosis and the memory estimate.
int cuju_b200_kernel_info(unsigned long long *out) {
    try {
        size_t local = 0, stack = 0;
        int regs = 0;
        cb::host::check(cb::kernel_attributes(&local, &regs), "kernel attributes");
        cb::host::check(cudaDeviceGetLimit(&stack, cudaLimitStackSize), "stack limit");
        out[0] = local;
        out[1] = (unsigned long long)regs;
        out[2] = stack;
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}

int cuju_state_padding(const char *bytes, unsigned long long size, unsigned char *mask) {
    try {
        if (!bytes || !mask) throw std::invalid_argument("expected the bytes of a match and a mask");
        cb::host::Codec codec;
        std::vector<size_t> positions;
        if (!codec.padding(std::string(bytes, size), positions))
            throw std::invalid_argument("expected the bytes of a match");
        memset(mask, 0, size);
        for (size_t p : positions) mask[p] = 1;
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}
const char *cuju_state_layout(unsigned long long *size) {
    if (size) *size = 0;
    lastError = "state layouts are not available in this backend";
    return nullptr;
}
int cuju_state_gather(const char *, unsigned long long, int, const unsigned long long *, const unsigned int *, int,
                      unsigned char *) {
    lastError = "state gathers are not available in this backend";
    return -1;
}

}  // extern "C"
#pragma GCC visibility pop
