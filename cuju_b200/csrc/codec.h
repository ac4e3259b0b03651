// cuju-b200 host: the GRF state bytes <-> Match. A state is the little-endian bytes of its fields
// in GRF's schema order (each struct's io() visits them in that order); lists are an int32 count
// then the elements; the team tactics are a count of (key, "%f" text) string pairs.
//   cuju include/cuju/state/archive.h:56-190 (Archive), environment_state.h:552-590 (tactics),
//   src/environment_state.cpp:11-100 (match and environment order),
//   include/cuju/simulation/state_io.h:20-90 (StateCodec: free-controller search, pointer checks,
//   frame conversion).
#pragma once

#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <memory>
#include <vector>

#include "match_util.cuh"

namespace cb {
namespace host {

constexpr int kMatchKeyboards = 22;

inline const char *tactic_key(int id) {
    static const char *const keys[kTactics] = {
        "position_defense_depth_factor",           "position_defense_microfocus_strength",
        "position_defense_midfieldfocus",          "position_defense_midfieldfocus_strength",
        "position_defense_ownhalf_factor",         "position_defense_sidefocus_strength",
        "position_defense_width_factor",           "position_offense_depth_factor",
        "position_offense_microfocus_strength",    "position_offense_midfieldfocus",
        "position_offense_midfieldfocus_strength", "position_offense_ownhalf_factor",
        "position_offense_sidefocus_strength",     "position_offense_width_factor"};
    return keys[id];
}

struct LoadedPointer {
    const int32_t *value;
    int kind;
};

// One cursor for both directions: `load` reads `bytes` into the fields, else appends the fields.
struct Archive {
    bool load;
    std::string bytes;
    size_t off = 0;
    std::vector<LoadedPointer> *pointers = nullptr;
    std::vector<size_t> *radians = nullptr;  // byte positions of the angles, when recorded

    template <class T>
    void f(T &v) {
        if (std::is_same<T, Radian>::value && radians) radians->push_back(off);
        if (load) {
            if (off + sizeof(T) > bytes.size()) throw std::runtime_error("state too short");
            memcpy(&v, bytes.data() + off, sizeof(T));
        } else {
            bytes.append(reinterpret_cast<const char *>(&v), sizeof(T));
        }
        off += sizeof(T);
    }
    void p(int32_t &v, int kind) {
        f(v);
        if (load && pointers) pointers->push_back({&v, kind});
    }
    template <class T, int N, class Fn>
    void vec(FVec<T, N> &v, Fn fn) {
        f(v.count);
        if (v.count < 0 || v.count > N) throw std::runtime_error("capacity exceeded");
        for (int i = 0; i < v.count; i++) fn(v.el[i]);
    }
    void str(std::string &s) {
        int32_t n = (int32_t)s.size();
        f(n);
        if (load) {
            if (n < 0 || (size_t)n > bytes.size() - off) throw std::runtime_error("state too short");
            s.assign(bytes.data() + off, (size_t)n);
            off += (size_t)n;
        } else {
            bytes.append(s);
            off += s.size();
        }
    }
    void check_team_sizes(int l, int r) {
        if (l < 0 || r < 0 || l > kTeamPlayers || r > kTeamPlayers)
            throw std::runtime_error("the state holds more players than a team holds");
    }
    void tactics(Tactics &t) {
        int32_t count = 0;
        for (int i = 0; i < kTactics; i++) count += (t.present >> i) & 1;
        f(count);
        if (load) {
            if (count < 0 || count > kTactics) throw std::runtime_error("properties: unexpected size");
            t.present = 0;
            for (int e = 0; e < count; e++) {
                std::string key, text;
                str(key);
                str(text);
                int id = 0;
                while (id < kTactics && key != tactic_key(id)) id++;
                if (id == kTactics) throw std::runtime_error("properties: unknown key " + key);
                char formatted[64];
                snprintf(formatted, sizeof(formatted), "%f", (double)(float)atof(text.c_str()));
                if (text != formatted) throw std::runtime_error("properties: value does not round-trip");
                t.present |= 1u << id;
                t.value[id] = (float)atof(text.c_str());
            }
        } else {
            for (int id = 0; id < kTactics; id++) {
                if (!((t.present >> id) & 1)) continue;
                std::string key = tactic_key(id);
                char formatted[64];
                snprintf(formatted, sizeof(formatted), "%f", (double)t.value[id]);
                std::string text = formatted;
                str(key);
                str(text);
            }
        }
    }
};

// The match, environment_state.cpp:11 (ProcessMatch).
inline void process_match(Archive &a, MatchState &m, int freeControllers) {
    a.f(m.firstTeam);
    a.f(m.secondTeam);
    a.vec(m.mentalImages, [&](MentalImage &im) { im.io(a); });
    m.teams[0].io(a);
    m.teams[1].io(a);
    for (int p = 0; p < m.playerCount; p++) m.players[p].io(a);
    a.f(m.goalCount[0]);
    a.f(m.goalCount[1]);
    a.f(m.possessionLastMinute);
    for (int o = 0; o < 3; o++) m.officials[o].io(a);
    // Every human gamer's keyboard a second time, first team first.
    const int kb = m.teams[0].gamers.count + m.teams[1].gamers.count;
    for (int k = 0; k < kb; k++) m.secondKeyboardCopies[k].io(a);
    m.freeControllerCount = freeControllers;
    for (int c = 0; c < freeControllers; c++) m.freeControllers[c].io(a);
    m.ball.io(a);
    a.f(m.matchTime_ms);
    a.f(m.actualTime_ms);
    a.f(m.goalScoredTimer);
    a.f(m.matchPhase);
    a.f(m.inPlay);
    a.f(m.inSetPiece);
    a.f(m.goalScored);
    a.f(m.ballIsInGoal);
    a.p(m.lastGoalTeam, kPtrTeam);
    a.p(m.lastGoalScorer, kPtrPlayer);
    for (int i = 0; i < 4; i++) a.f(m.lastTouchTeamIDs[i]);
    a.f(m.lastTouchTeamID);
    a.p(m.bestPossessionTeam, kPtrTeam);
    a.p(m.designatedPossessionPlayer, kPtrPlayer);
    a.p(m.ballRetainer, kPtrPlayer);
    a.f(m.possessionSideHistoryMaxTime_ms);
    a.vec(m.possessionSideHistory, [&](float &v) { a.f(v); });
    a.f(m.autoUpdateInGameCamera);
    a.f(m.cameraOrientation);
    a.f(m.cameraNodeOrientation);
    a.f(m.cameraNodePosition);
    a.f(m.cameraFieldOfView);
    a.f(m.cameraNearCap);
    a.f(m.cameraFarCap);
    a.vec(m.cameraPosition, [&](Vec3 &v) { a.f(v); });
    a.f(m.lastBodyBallCollisionTime_ms);
    m.referee.io(a);
}

// The start of a state up to its scenario, then the step and the match
// (environment_state.cpp:74-100).
inline void process_scenario(Archive &a, Match &w) {
    a.f(w.gameState);
    a.f(w.waitingForGameCount);
    for (int i = 0; i < 2512; i++) a.f(w.rng[i]);
    w.scenario.io(a);
}
inline void process_state(Archive &a, Match &w, int freeControllers) {
    process_scenario(a, w);
    w.m.playerCount = w.scenario.leftTeamSize + w.scenario.rightTeamSize;
    if (w.m.playerCount > kPlayers) throw std::runtime_error("the state holds more players than a match holds");
    a.f(w.step);
    process_match(a, w.m, freeControllers);
}

// A default world: all zero, both teams on side -1 in their own frame.
inline void clear_match(Match &w) {
    memset(static_cast<void *>(&w), 0, sizeof(Match));
    w.flags.teamSide[0] = -1;
    w.flags.teamSide[1] = -1;
}

// A state does not record its free-controller count, so a codec finds it on the first load and
// tries it first afterwards (state_io.h:20).
struct Codec {
    int freeControllerCount = -1;
    int animationCount = -1;  // -1 leaves animation pointers unchecked

    bool pointers_in_range(const Match &w, const std::vector<LoadedPointer> &ps) const {
        const MatchState &m = w.m;
        const int sizes[5] = {m.playerCount, 2, m.teams[0].gamers.count + m.teams[1].gamers.count,
                              kMatchKeyboards, animationCount};
        for (const LoadedPointer &p : ps) {
            const int n = sizes[p.kind];
            if (n >= 0 && (*p.value < -1 || *p.value >= n)) return false;
        }
        return true;
    }
    bool load(const std::string &bytes, Match &w) {
        auto attempt = [&](int fc) {
            try {
                clear_match(w);
                std::vector<LoadedPointer> ps;
                Archive a{true, bytes};
                a.pointers = &ps;
                process_state(a, w, fc);
                return a.off == a.bytes.size() && pointers_in_range(w, ps);
            } catch (const std::exception &) {
                return false;
            }
        };
        if (freeControllerCount >= 0 && attempt(freeControllerCount)) return true;
        for (int fc = 0; fc <= kControllers; fc++)
            if (attempt(fc)) {
                freeControllerCount = fc;
                return true;
            }
        return false;
    }
    std::string save(Match &w) {
        ball_materialize(w.m.ball);
        for (int i = 0; i < w.m.mentalImages.count; i++) mental_materialize(w.m.mentalImages.el[i]);
        Archive a{false, std::string()};
        process_state(a, w, freeControllerCount);
        return a.bytes;
    }
    // state_api.h:21 (cuju_state_padding): GRF saves an angle as its float, its flag and three
    // bytes of padding that hold whatever its memory held; the positions of those bytes in the
    // match bytes, so that two states can be compared without them. Empty if the bytes hold no
    // match.
    bool padding(const std::string &bytes, std::vector<size_t> &positions) {
        std::unique_ptr<Match> w(new Match);
        if (!load(bytes, *w)) return false;
        std::vector<size_t> radians;
        Archive a{true, bytes};
        a.radians = &radians;
        clear_match(*w);
        process_state(a, *w, freeControllerCount);
        positions.clear();
        for (size_t r : radians)
            if (r + 8 <= bytes.size())
                for (size_t k = 5; k < 8; k++) positions.push_back(r + k);
        return true;
    }
    // Bytes to a world in the rest frame (mirror 0), as StateCodec::LoadFrame.
    bool load_frame(const std::string &bytes, Match &w) {
        if (!load(bytes, w)) return false;
        init_player_teams(w);
        canonical_to_rest(w);
        return true;
    }
    // A world in the rest frame to bytes; the world is left as it was.
    std::string save_frame(Match &w) {
        canonical_to_rest(w);
        std::string b = save(w);
        canonical_to_rest(w);
        return b;
    }
};

}  // namespace host
}  // namespace cb
