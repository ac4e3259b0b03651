// cuju-b200: how the lanes of a warp share the rare, long branches of a tick, and how the warps of
// an SM move through a tick together.
//
// The step is bound by the SM's instruction cache, not by arithmetic or memory bandwidth: the
// kernel is megabytes of code, and warps of one SM that run different parts of it evict each
// other's lines. Two mechanisms keep lanes and warps on the same code:
//
// * Assist rounds. A humanoid's interrupt branch (command request and animation selection), its
//   touch branch and an official's interrupt branch are rare per environment but long, and wide
//   inside (filters over ~1,500 animations, candidate sorts). When the 32 lanes of a warp of crews
//   of one reach one together, the environments that need it are dealt to crews of the warp
//   (crew.cuh), which run the branch and divide its wide loops between their lanes, instead of
//   one lane running it while the others wait.
// * Convoy. At a waypoint (the start of a tick, of each of its phases, of each player's turn and of
//   a humanoid's interrupt and touch branches) a warp whose 32 lanes arrive together waits, a
//   bounded number of times, until every
//   lane of the block's other warps has reached that point of its own match or finished. A lane's
//   place is a key: ticks run in this call, then the waypoint's rank within the tick.
//
// Neither changes what a match computes: a branch reads and writes only its environment's memory
// and returns its result to the lane that owns the environment; waits only decide when a warp
// issues its next instruction. Every wait is bounded.
#pragma once

#include "crew.cuh"
#include "sim.cuh"

namespace cb {

enum AssistJob { kJobInterrupt = 1, kJobTouches = 2, kJobOfficialInterrupt = 3 };
// Runs an assisted branch for the environment of `s` (defined after the branches, in officials.cuh).
CB_HDNI bool assist_job(const Sim &s, int kind, int arg);

constexpr int kAssistCrewsMax = 8;          // crews of 4 lanes at the narrowest
constexpr unsigned kConvoyDone = 0xffffffffu;
constexpr int kConvoySpins = 2000;          // naps a waypoint waits at most
constexpr unsigned kNapNs = 100;

__device__ __forceinline__ unsigned *convoy_keys() {
    __shared__ unsigned keys[kCrewSlots];
    return keys;
}
__device__ __forceinline__ unsigned *convoy_ticks() {
    __shared__ unsigned ticks[kCrewSlots];
    return ticks;
}
// Every thread of the block calls this once, before any returns: lanes without an environment
// count as finished.
__device__ __forceinline__ void convoy_start(bool live) {
    convoy_keys()[threadIdx.x] = live ? 0u : kConvoyDone;
    convoy_ticks()[threadIdx.x] = 0;
    __syncthreads();
}
// A lane that has finished its call.
__device__ __forceinline__ void convoy_leave() { ((volatile unsigned *)convoy_keys())[threadIdx.x] = kConvoyDone; }

// Runs assist_job(s, kind, arg) for the environment of every lane whose `need` is set, and returns
// the calling lane's result (true where not needed). When the 32 lanes of a warp of crews of one
// reach the call together, the k environments that need it are dealt to crews: c crews of 32/c
// lanes, c the smallest power of two at least k (at most kAssistCrewsMax), in rounds of c
// environments. Otherwise every lane makes its own call. The branch reads and writes only device
// memory reachable from the Sim it is given, never the calling lane's locals. The result and any
// iteration-cap mark of an environment go back to the lane that owns it.
CB_HD bool crew_assist(const Sim &s, int kind, int arg, bool need) {
#if CB_DEVICE_PASS
    if (crew_owns_env() && __activemask() == 0xffffffffu) {
        const unsigned full = 0xffffffffu;
        const unsigned pending = __ballot_sync(full, need);
        if (!pending) return true;
        const int k = __popc(pending);
        int log2c = 0;
        while ((1 << log2c) < k && (1 << log2c) < kAssistCrewsMax) log2c++;
        const int crews = 1 << log2c, log2w = 5 - log2c, width = 1 << log2w;
        const unsigned widthBits = width == 32 ? full : (1u << width) - 1u;
        const int lane = lane_id();
        const int crew = lane >> log2w;
        const int myPlace = __popc(pending & ((1u << lane) - 1u));
        const bool ownCap = crew_cap_reached();
        bool mine = true, myCap = false;
        for (int first = 0; first < k; first += crews) {
            // The environment this lane's crew runs in this round: the (first + crew)-th that needs it.
            const int place = first + crew;
            unsigned rest = pending;
            for (int i = 0; i < place && rest; i++) rest &= rest - 1;
            const int src = place < k ? __ffs(rest) - 1 : lane;
            Match *wp = reinterpret_cast<Match *>(
                __shfl_sync(full, reinterpret_cast<unsigned long long>(&s.w), src));
            const Context *cp = reinterpret_cast<const Context *>(
                __shfl_sync(full, reinterpret_cast<unsigned long long>(&s.ctx), src));
            WarpScratch *sp = reinterpret_cast<WarpScratch *>(
                __shfl_sync(full, reinterpret_cast<unsigned long long>(s.scratch), src));
            int32_t *stp = reinterpret_cast<int32_t *>(
                __shfl_sync(full, reinterpret_cast<unsigned long long>(s.status), src));
            const int a = __shfl_sync(full, arg, src);
            __syncwarp(full);
            crew_clear_cap();
            bool r = true;
            if (place < k) {
                crew_set(log2w);
                const Sim shared{*wp, *cp, sp, stp};
                r = assist_job(shared, kind, a);
                crew_set(0);
            }
            __syncwarp(full);
            const unsigned caps = __ballot_sync(full, crew_cap_reached());
            const bool served = need && myPlace >= first && myPlace < first + crews;
            const int from = served ? (myPlace - first) << log2w : lane;
            const int got = __shfl_sync(full, (int)r, from);
            if (served) {
                mine = got != 0;
                myCap = ((caps >> from) & widthBits) != 0;
            }
        }
        crew_clear_cap();
        if (ownCap || myCap) crew_note_cap();
        return mine;
    }
#endif
    return need ? assist_job(s, kind, arg) : true;
}

// Waypoint ranks, in the order a tick reaches them: the ball and referee phases, each team's turn
// (its team AI, then per player: the turn, the interrupt branch, the touch branch), and the phases
// after both teams. A lane skips the ranks of phases its match does not run this tick.
constexpr unsigned kWayBallCollisions = 1, kWayBallProcess = 2, kWaySwitch = 3;
CB_HD constexpr unsigned way_team(int slot) { return 4u + 72u * (unsigned)slot; }
CB_HD constexpr unsigned way_player(int slot, int p, int part) { return way_team(slot) + 1u + 3u * (unsigned)p + (unsigned)part; }
constexpr unsigned kWayOfficials = 150, kWayPossession = 151, kWayCollisions = 153, kWayCamera = 154,
                   kWayPrepare = 155, kWayFetch = 156;
static_assert(way_player(1, kPlayers - 1, 2) < kWayOfficials, "ranks increase through a tick");

// A waypoint of rank `rank` (1-255, increasing through a tick).
CB_HD void convoy_waypoint(unsigned rank) {
#if CB_DEVICE_PASS && __CUDA_ARCH__ >= 800
    if (!crew_owns_env()) return;
    volatile unsigned *keys = convoy_keys();
    const unsigned key = (convoy_ticks()[threadIdx.x] << 8) | rank;
    keys[threadIdx.x] = key;
    if (__activemask() != 0xffffffffu) return;
    const unsigned mine = __reduce_min_sync(0xffffffffu, key);
    const int w = (int)(threadIdx.x >> 5), warps = (int)(blockDim.x >> 5), l = lane_id();
    for (int spin = 0; spin < kConvoySpins; spin++) {
        bool behind = false;
        for (int o = 0; o < warps; o++)
            if (o != w && keys[o * 32 + l] < mine) behind = true;
        if (!__any_sync(0xffffffffu, behind)) break;
        __nanosleep(kNapNs);
    }
#else
    (void)rank;
#endif
}
// The start of a tick.
CB_HD void convoy_tick() {
#if CB_DEVICE_PASS && __CUDA_ARCH__ >= 800
    if (!crew_owns_env()) return;
    convoy_ticks()[threadIdx.x]++;
    convoy_waypoint(0);
#endif
}

}  // namespace cb
