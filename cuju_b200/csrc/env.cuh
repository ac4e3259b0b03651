// cuju-b200: GRF's environment on top of the ticks — actions, keyboards, the observation, the
// episode rules, agent views, simple115 and the checkpoint reward, and one environment's reset and
// step inside a batch.
//   cuju include/cuju/simulation/environment.h:17-590
//   cuju include/cuju/simulation/observation_encoding.h:16-180
//   cuju include/cuju/batch/batch_core.h:262-649
#pragma once

#include "match.cuh"

namespace cb {

enum Action {
    kActIdle = 0, kActLeft, kActTopLeft, kActTop, kActTopRight, kActRight, kActBottomRight, kActBottom,
    kActBottomLeft, kActLongPass, kActHighPass, kActShortPass, kActShot, kActKeeperRush, kActSliding,
    kActPressure, kActTeamPressure, kActSwitch, kActSprint, kActDribble, kActReleaseDirection,
    kActReleaseLongPass, kActReleaseHighPass, kActReleaseShortPass, kActReleaseShot, kActReleaseKeeperRush,
    kActReleaseSliding, kActReleasePressure, kActReleaseTeamPressure, kActReleaseSwitch, kActReleaseSprint,
    kActReleaseDribble, kActBuiltinAI
};

/// environment.h:56-96: action sets 0 `default` (19), 1 `v2` (20), 2 `full` (33), each a prefix of
/// the full list.
CB_HD int action_set_size(int set) { return set == 0 ? 19 : set == 1 ? 20 : 33; }
CB_HD int action_from_set(int index) {
    switch (index) {
        case 0: return kActIdle;
        case 1: return kActLeft;
        case 2: return kActTopLeft;
        case 3: return kActTop;
        case 4: return kActTopRight;
        case 5: return kActRight;
        case 6: return kActBottomRight;
        case 7: return kActBottom;
        case 8: return kActBottomLeft;
        case 9: return kActLongPass;
        case 10: return kActHighPass;
        case 11: return kActShortPass;
        case 12: return kActShot;
        case 13: return kActSprint;
        case 14: return kActReleaseDirection;
        case 15: return kActReleaseSprint;
        case 16: return kActSliding;
        case 17: return kActDribble;
        case 18: return kActReleaseDribble;
        case 19: return kActBuiltinAI;
        case 20: return kActKeeperRush;
        case 21: return kActPressure;
        case 22: return kActTeamPressure;
        case 23: return kActSwitch;
        case 24: return kActReleaseLongPass;
        case 25: return kActReleaseHighPass;
        case 26: return kActReleaseShortPass;
        case 27: return kActReleaseShot;
        case 28: return kActReleaseKeeperRush;
        case 29: return kActReleaseSliding;
        case 30: return kActReleasePressure;
        case 31: return kActReleaseTeamPressure;
        default: return kActReleaseSwitch;
    }
}

enum { kNegateX = 1, kNegateY = 2 };
/// environment.h:101: the action pointing the same way on a pitch whose x and/or y change sign.
CB_HD int negate_action_axes(int a, bool nx, bool ny) {
    int h, v;
    switch (a) {
        case kActLeft: h = -1, v = 0; break;
        case kActTopLeft: h = -1, v = -1; break;
        case kActTop: h = 0, v = -1; break;
        case kActTopRight: h = 1, v = -1; break;
        case kActRight: h = 1, v = 0; break;
        case kActBottomRight: h = 1, v = 1; break;
        case kActBottom: h = 0, v = 1; break;
        case kActBottomLeft: h = -1, v = 1; break;
        default: return a;
    }
    if (nx) h = -h;
    if (ny) v = -v;
    if (v == -1) return h == -1 ? kActTopLeft : h == 0 ? kActTop : kActTopRight;
    if (v == 1) return h == -1 ? kActBottomLeft : h == 0 ? kActBottom : kActBottomRight;
    return h == -1 ? kActLeft : h == 0 ? a : kActRight;
}

constexpr int kMaxSticky = 13;
CB_HD int sticky_count(int set) { return set == 2 ? 13 : 10; }
CB_HD int sticky_action(int i) {
    switch (i) {
        case 0: return kActLeft;
        case 1: return kActTopLeft;
        case 2: return kActTop;
        case 3: return kActTopRight;
        case 4: return kActRight;
        case 5: return kActBottomRight;
        case 6: return kActBottom;
        case 7: return kActBottomLeft;
        case 8: return kActSprint;
        case 9: return kActDribble;
        case 10: return kActKeeperRush;
        case 11: return kActPressure;
        default: return kActTeamPressure;
    }
}

constexpr int kTeamControllers = 11;
constexpr int kAgentsMax = 2 * kTeamControllers;

// The state holds a gamer's keyboard twice (in the gamer and among the match's second copies), a
// free controller once (free controllers are those no gamer owns, in ID order), some none at all.
// environment.h:155 (Keyboard).
struct KeyboardCopies {
    Keyboard *k[2];
    int n;
};
CB_HDNI KeyboardCopies keyboard_copies(Match &w, int cid) {
    MatchState &m = w.m;
    KeyboardCopies r;
    r.n = 0;
    const int gc = m.teams[0].gamers.count + m.teams[1].gamers.count;
    for (int g = 0; g < gc; g++) {
        if (gamer_global(w, g).keyboardIndex == cid) {
            r.k[0] = &gamer_global(w, g).controller.keyboard;
            r.k[1] = &m.secondKeyboardCopies[g];
            r.n = 2;
            return r;
        }
    }
    int fi = 0;
    for (int c = 0; c < cid; c++) {
        bool owned = false;
        for (int g = 0; g < gc; g++) owned |= gamer_global(w, g).keyboardIndex == c;
        if (!owned) fi++;
    }
    if (fi < m.freeControllerCount) {
        r.k[0] = &m.freeControllers[fi];
        r.n = 1;
    }
    return r;
}

/// environment.h:180 (EnvironmentAction); `player` indexes the agent within its team.
CB_HDNI void environment_action(Match &w, int action, bool left, int player) {
    KeyboardCopies kc = keyboard_copies(w, player + (left ? 0 : kTeamControllers));
    for (int i = 0; i < kc.n; i++) {
        Keyboard *kb = kc.k[i];
        // A state holds a keyboard's direction times its mirror sign.
        auto dir = [&](float x, float y) { kb->direction = Vec3(x, y, 0) * kb->mirror; };
        auto btn = [&](int b, bool p) { kb->buttons[b] = p; };
        kb->disabled = false;
        switch (action) {
            case kActLeft: dir(-1, 0); break;
            case kActTopLeft: dir(-1, 1); break;
            case kActTop: dir(0, 1); break;
            case kActTopRight: dir(1, 1); break;
            case kActRight: dir(1, 0); break;
            case kActBottomRight: dir(1, -1); break;
            case kActBottom: dir(0, -1); break;
            case kActBottomLeft: dir(-1, -1); break;
            case kActLongPass: btn(kBtnLongPass, true); break;
            case kActHighPass: btn(kBtnHighPass, true); break;
            case kActShortPass: btn(kBtnShortPass, true); break;
            case kActShot: btn(kBtnShot, true); break;
            case kActKeeperRush: btn(kBtnKeeperRush, true); break;
            case kActSliding: btn(kBtnSliding, true); break;
            case kActPressure: btn(kBtnPressure, true); break;
            case kActTeamPressure: btn(kBtnTeamPressure, true); break;
            case kActSwitch: btn(kBtnSwitch, true); break;
            case kActSprint: btn(kBtnSprint, true); break;
            case kActDribble: btn(kBtnDribble, true); break;
            case kActReleaseDirection: dir(0, 0); break;
            case kActReleaseLongPass: btn(kBtnLongPass, false); break;
            case kActReleaseHighPass: btn(kBtnHighPass, false); break;
            case kActReleaseShortPass: btn(kBtnShortPass, false); break;
            case kActReleaseShot: btn(kBtnShot, false); break;
            case kActReleaseKeeperRush: btn(kBtnKeeperRush, false); break;
            case kActReleaseSliding: btn(kBtnSliding, false); break;
            case kActReleasePressure: btn(kBtnPressure, false); break;
            case kActReleaseTeamPressure: btn(kBtnTeamPressure, false); break;
            case kActReleaseSwitch: btn(kBtnSwitch, false); break;
            case kActReleaseSprint: btn(kBtnSprint, false); break;
            case kActReleaseDribble: btn(kBtnDribble, false); break;
            case kActBuiltinAI:
                // Disabling zeroes the direction (times the mirror sign: a right keyboard holds -0).
                kb->disabled = true;
                dir(0, 0);
                for (int b = 0; b < kBtnCount; b++) kb->buttons[b] = false;
                break;
            default: break;
        }
    }
}

/// environment.h:298 (StickyActionState): a controller the state does not hold is at rest.
CB_HDNI bool sticky_action_state(Match &w, int action, bool left, int player) {
    KeyboardCopies kc = keyboard_copies(w, player + (left ? 0 : kTeamControllers));
    if (kc.n == 0) return false;
    const Keyboard &kb = *kc.k[0];
    const Vec3 d = kb.direction * kb.mirror;
    auto is = [&](float x, float y) { return d.c[0] == x && d.c[1] == y && d.c[2] == 0.0f; };
    switch (action) {
        case kActLeft: return is(-1, 0);
        case kActTopLeft: return is(-1, 1);
        case kActTop: return is(0, 1);
        case kActTopRight: return is(1, 1);
        case kActRight: return is(1, 0);
        case kActBottomRight: return is(1, -1);
        case kActBottom: return is(0, -1);
        case kActBottomLeft: return is(-1, -1);
        case kActKeeperRush: return kb.buttons[kBtnKeeperRush];
        case kActPressure: return kb.buttons[kBtnPressure];
        case kActTeamPressure: return kb.buttons[kBtnTeamPressure];
        case kActSprint: return kb.buttons[kBtnSprint];
        case kActDribble: return kb.buttons[kBtnDribble];
        default: return false;
    }
}

// After a step in play, the non-sticky buttons of every controller release (environment.h:337).
CB_HDNI void release_step_buttons(Match &w) {
    for (int c = 0; c < 2 * kTeamControllers; c++) {
        KeyboardCopies kc = keyboard_copies(w, c);
        for (int i = 0; i < kc.n; i++) {
            bool *b = kc.k[i]->buttons;
            b[kBtnLongPass] = b[kBtnHighPass] = b[kBtnShortPass] = b[kBtnShot] = b[kBtnSliding] = b[kBtnSwitch] =
                false;
        }
    }
}
CB_HDNI bool environment_step(const Sim &s) {
    for (int t = 0; t < s.ctx.ticksPerStep; t++)
        if (!game_tick(s)) return false;
    if (s.w.m.inPlay) {
        s.w.step++;
        release_step_buttons(s.w);
    }
    return true;
}

// Observation coordinates: x and y divide in double by GRF's field scales, z by the integer 1.
CB_HD float env_coord(const Vec3 &v, int i) {
    if (i == 0) return (float)((double)v.c[0] / 54.4);
    if (i == 1) return (float)((double)v.c[1] / -83.6);
    return v.c[2] / 1;
}

struct PlayerObs {
    float position[2], direction[2];
    float tiredFactor;
    bool active, yellowCard;
    int32_t role;
};
struct TeamObs {
    int32_t count;
    PlayerObs players[kTeamPlayers];
    int32_t designatedPlayer;
};
// GRF's observation from the left team's side; team[0] is the left team; player indices count
// within a team and -1 marks none (environment.h:361-384).
struct Observation {
    float ball[3], ballDirection[3], ballRotation[3];
    TeamObs team[2];
    int32_t controlledPlayer[2][kTeamControllers];
    int32_t gameMode;
    int32_t score[2];
    int32_t ballOwnedTeam, ballOwnedPlayer;
    int32_t step;
    bool isInPlay;
};

/// environment.h:387 (EnvironmentGetState).
CB_HDNI void environment_get_state(Match &w, const Context &ctx, Observation &o) {
    const MatchState &m = w.m;
    crew_copy_words(reinterpret_cast<uint32_t *>(&o), nullptr, (int)(sizeof(Observation) / 4));
    o.team[0].designatedPlayer = -1;
    o.team[1].designatedPlayer = -1;
    auto set3 = [](float *out, const Vec3 &v) {
        for (int i = 0; i < 3; i++) out[i] = env_coord(v, i);
    };
    set3(o.ball, ball_average_position(w, 5));
    float rx, ry, rz;
    m.ball.rotationPerMs.angles(rx, ry, rz);
    set3(o.ballRotation, Vec3(rx, ry, rz) / (float)ctx.ticksPerStep);
    set3(o.ballDirection, m.ball.momentum / (float)ctx.ticksPerStep);
    o.ballOwnedPlayer = -1;
    o.ballOwnedTeam = -1;
    o.score[0] = goal_count(w, 0);
    o.score[1] = goal_count(w, 1);
    // The step before the start at 2000 ms, which ends at 1900 ms, reports in play.
    o.isInPlay = m.inPlay || m.actualTime_ms == 1900;
    o.gameMode = m.inSetPiece ? m.referee.buffer.desiredSetPiece : kGmNormal;
    for (int t = 0; t < 2; t++)
        for (int c = 0; c < kTeamControllers; c++) o.controlledPlayer[t][c] = -1;
    const int first = w.firstTeamID();
    for (int k = 0; k < 2; k++) {
        const int teamID = k == 0 ? first : 1 - first;
        TeamObs &to = o.team[teamID];
        const Team &team = team_by_id(w, teamID);
        PlayerList ps;
        all_players(ps, w, teamID);
        for (int i = 0; i < ps.count; i++) {
            const int p = ps[i];
            const Player &pl = m.players[p];
            if (pl.base.externalController >= 0) {
                int c = gamer_global(w, pl.base.externalController).keyboardIndex;
                o.controlledPlayer[teamID][c % kTeamControllers] = to.count;
            }
            Vec3 pos = pl.base.humanoid.spatial.position;
            Vec3 mv = pl.base.humanoid.spatial.movement;
            if (teamID == 1) {
                pos.mirror();
                mv.mirror();
            }
            PlayerObs &po = to.players[to.count];
            po.position[0] = env_coord(pos, 0);
            po.position[1] = env_coord(pos, 1);
            Vec3 d = mv / (float)ctx.ticksPerStep;
            po.direction[0] = env_coord(d, 0);
            po.direction[1] = env_coord(d, 1);
            po.tiredFactor = 1 - pl.base.fatigueFactorInverse;
            po.yellowCard = pl.cards > 0;
            po.active = pl.base.isActive;
            po.role = ctx.staticData->formation[formation_source(w, p)].role;
            if (pl.hasPossession && m.lastTouchTeamID != -1 &&
                team_by_id(w, match_last_touch_team(w)).lastTouchPlayer == p) {
                o.ballOwnedPlayer = to.count;
                o.ballOwnedTeam = m.lastTouchTeamID;
            }
            if (p == team.mainSelectedPlayer) to.designatedPlayer = to.count;
            to.count++;
        }
    }
    o.step = w.step;
}

enum { kGsCreated, kGsInitiated, kGsRunning, kGsDone };

/// environment.h:465 (EnvironmentResetFromTemplate): `w` holds a copy of the template (the state
/// after a reset of the same scenario, agents and team order); other seeds differ only in the RNG,
/// the stored seed and the humanoids' idle frames, so this reseeds and replays the reset draws.
CB_HDNI bool reset_from_template(const Sim &s, uint32_t seed) {
    Match &w = s.w;
    w.scenario.gameEngineRandomSeed = seed;
    MatchRng{w.rng}.seed(seed);
    const int pc = w.m.playerCount;
    for (int p = 0; p < pc; p++) {
        const int side = team_side(w, w.playerTeamID[p]);
        if (!humanoid_reset_position(s, p, Vec3(0), Vec3(0))) return false;
        Vec3 pos = formation(s, p).position * 25 * Vec3(-side, -side, 0);
        if (!humanoid_reset_position(s, p, pos, Vec3(0))) return false;
    }
    random_in_range(w.rng, 1, 4);  // the officials' skin colour
    for (int o = 0; o < 3; o++)
        for (int d = 0; d < 2; d++)
            if (!humanoid_reset_position(s, pc + o, Vec3(0), Vec3(0))) return false;
    const Vec3 placed[3] = {Vec3(10, -10, 0), Vec3(25, -36.5f, 0), Vec3(-25, 36.5f, 0)};
    for (int o = 0; o < 3; o++)
        if (!humanoid_reset_position(s, pc + o, placed[o], Vec3(0))) return false;
    // The lighting draws six times and affects nothing else.
    random_in_range(w.rng, -1.7f, 1.7f);
    random_in_range(w.rng, -1.7f, 1.7f);
    random_in_range(w.rng, 0, 1);
    for (int d = 0; d < 3; d++) random_in_range(w.rng, (float)-0.1, (float)0.1);
    return true;
}

// A restart waits at most a card's 12 s stoppage plus the set-piece preparation (about 150 steps);
// a state that waits longer is malformed, and the bound keeps a step finite.
constexpr int kMaxWaitSteps = 2000;

struct EnvCore {
    int32_t previousScoreDifference;
    int32_t previousGameMode;
    int32_t previousBallOwnedTeam;
    Observation observation;
};

// Ticks until the match is in play (environment.h:582, EnvironmentCoreAfterReset).
CB_HDNI bool core_after_reset(const Sim &s, EnvCore &core) {
    core.previousScoreDifference = 0;
    core.previousGameMode = -1;
    core.previousBallOwnedTeam = -1;
    // A reset reaches play within seconds; the bound only guards a malformed template.
    for (int guard = 0; guard < kMaxWaitSteps; guard++) {
        environment_get_state(s.w, s.ctx, core.observation);
        if (core.observation.isInPlay) return true;
        if (!environment_step(s)) return false;
    }
    return s.fail(kStatusUnsupported);
}

/// environment.h:512 (EnvironmentCoreStep): `actions` one per agent, left agents first; `reward`
/// the left team's change of score difference. After 20 steps in a set piece every agent
/// short-passes, then the ball owner's agent runs to one side and back while the rest idle.
CB_HDNI bool core_step(const Sim &s, EnvCore &core, const int *actions, int &reward, bool &done) {
    Match &w = s.w;
    const Scenario &sc = w.scenario;
    int ai = 0;
    for (int side = 0; side < 2; side++) {
        const bool left = side == 0;
        const int agents = left ? sc.leftAgents : sc.rightAgents;
        for (int a = 0; a < agents; a++) {
            int act = actions[ai];
            if (w.waitingForGameCount == 20) {
                act = kActShortPass;
            } else if (w.waitingForGameCount > 20) {
                act = kActIdle;
                const int controlled = core.observation.controlledPlayer[left ? 0 : 1][a];
                if (core.observation.ballOwnedTeam != -1 && (core.observation.ballOwnedTeam ^ (int)left) &&
                    controlled == core.observation.ballOwnedPlayer) {
                    if ((w.waitingForGameCount < 30) != left) act = kActLeft;
                    else act = kActRight;
                }
            }
            ai++;
            environment_action(w, act, left, a);
        }
    }
    // Play resumes within seconds of game time; the bound only guards a malformed state.
    for (int guard = 0;; guard++) {
        if (guard > kMaxWaitSteps) return s.fail(kStatusUnsupported);
        for (int t = 0; t < s.ctx.ticksPerStep; t++)
            if (!game_tick(s)) return false;
        if (w.m.inPlay) {
            w.step++;
            release_step_buttons(w);
        }
        environment_get_state(w, s.ctx, core.observation);
        if (core.observation.isInPlay) break;
    }
    const Observation &o = core.observation;
    if (sc.endEpisodeOnScore && (o.score[0] > 0 || o.score[1] > 0)) w.gameState = kGsDone;
    if (sc.endEpisodeOnOutOfPlay && o.gameMode != kGmNormal && core.previousGameMode == kGmNormal)
        w.gameState = kGsDone;
    core.previousGameMode = o.gameMode;
    if (sc.endEpisodeOnPossessionChange && o.ballOwnedTeam != -1 && core.previousBallOwnedTeam != -1 &&
        o.ballOwnedTeam != core.previousBallOwnedTeam)
        w.gameState = kGsDone;
    if (o.ballOwnedTeam != -1) core.previousBallOwnedTeam = o.ballOwnedTeam;
    const int diff = o.score[0] - o.score[1];
    reward = diff - core.previousScoreDifference;
    core.previousScoreDifference = diff;
    if (o.gameMode != kGmNormal) w.waitingForGameCount += 1;
    else w.waitingForGameCount = 0;
    if (o.step >= sc.gameDuration) w.gameState = kGsDone;
    done = w.gameState == kGsDone;
    return true;
}

// ---------------------------------------------------------------------------------------------
// Agent views and encodings (observation_encoding.h).

// The agent's own team is team[0]; `active` and `designated` index it (-1 for none).
struct AgentView {
    Observation o;
    int active, designated, stickyCount;
    uint8_t sticky[kMaxSticky];
};

CB_HD void make_agent_view(const Observation &raw, bool right, int agent, int actionSet, const uint8_t *sticky,
                           AgentView &v) {
    v.o = raw;
    if (right) {
        // The right team's side: teams, scores and controllers swap (SwapTeams).
        v.o.ballOwnedTeam = raw.ballOwnedTeam > -1 ? 1 - raw.ballOwnedTeam : -1;
        v.o.score[0] = raw.score[1];
        v.o.score[1] = raw.score[0];
        for (int t = 0; t < 2; t++) {
            v.o.team[t] = raw.team[1 - t];
            for (int c = 0; c < kTeamControllers; c++) v.o.controlledPlayer[t][c] = raw.controlledPlayer[1 - t][c];
        }
        // Both axes negate for a right agent (NegateGeometry).
        for (int k = 0; k < 2; k++) {
            v.o.ball[k] = -v.o.ball[k];
            v.o.ballDirection[k] = -v.o.ballDirection[k];
        }
        for (int t = 0; t < 2; t++)
            for (int p = 0; p < v.o.team[t].count; p++)
                for (int k = 0; k < 2; k++) {
                    v.o.team[t].players[p].position[k] = -v.o.team[t].players[p].position[k];
                    v.o.team[t].players[p].direction[k] = -v.o.team[t].players[p].direction[k];
                }
    }
    v.designated = v.o.team[0].designatedPlayer;
    v.active = v.o.controlledPlayer[0][agent];
    v.stickyCount = sticky_count(actionSet);
    // Entry i takes the state of the sticky action that points its way on the agent's pitch.
    for (int i = 0; i < v.stickyCount; i++) {
        int src = i;
        if (right) {
            const int flipped = negate_action_axes(sticky_action(i), true, true);
            for (int o = 0; o < v.stickyCount; o++)
                if (sticky_action(o) == flipped) src = o;
        }
        v.sticky[i] = sticky[src];
    }
}

/// observation_encoding.h:92 (EncodeSimple115): left positions, left directions, right positions,
/// right directions (22 values each when `fixed`, as simple115v2), ball, ball direction, one-hots
/// of owning team (3), active player (11) and game mode (7); missing values -1.
CB_HDNI void encode_simple115(const AgentView &v, bool fixed, float *out) {
    int n = 0;
    for (int part = 0; part < 4; part++) {
        const TeamObs &t = v.o.team[part / 2];
        const bool dirs = part % 2 == 1;
        for (int p = 0; p < t.count; p++)
            for (int k = 0; k < 2; k++) out[n++] = dirs ? t.players[p].direction[k] : t.players[p].position[k];
        if (fixed)
            while (n < (part + 1) * 22) out[n++] = -1;
    }
    while (n < 88) out[n++] = -1;
    for (int i = 0; i < 3; i++) out[n++] = v.o.ball[i];
    for (int i = 0; i < 3; i++) out[n++] = v.o.ballDirection[i];
    for (int i = 0; i < 3; i++) out[n++] = (v.o.ballOwnedTeam + 1 == i) ? 1.0f : 0.0f;
    for (int i = 0; i < 11; i++) out[n++] = (v.active != -1 && v.active == i) ? 1.0f : 0.0f;
    for (int i = 0; i < 7; i++) out[n++] = (v.o.gameMode == i) ? 1.0f : 0.0f;
}

// numpy's type promotion: before numpy 2 (legacy) the sum runs in double and rounds to float;
// from numpy 2 on the increment rounds to float and the sum runs in float.
CB_HD float add_float(float r, double inc, bool legacy) { return legacy ? (float)((double)r + inc) : r + (float)inc; }
/// observation_encoding.h:157 (CheckpointReward).
CB_HDNI float checkpoint_reward(const AgentView &v, float reward, int &collected, bool legacy) {
    const int cc = 10;
    const double cr = 0.1;
    if (reward == 1) {
        reward = add_float(reward, cr * (cc - collected), legacy);
        collected = cc;
        return reward;
    }
    if (v.o.ballOwnedTeam != 0 || v.o.ballOwnedPlayer != v.active) return reward;
    const float bx = v.o.ball[0], by = v.o.ball[1];
    const double d = lm::lm_pow(lm::lm_pow((double)bx - 1, 2.0) + lm::lm_pow((double)by, 2.0), 0.5);
    while (collected < cc) {
        const double thr = 0.99 - 0.8 / (cc - 1) * collected;
        if (d > thr) break;
        reward = add_float(reward, cr, legacy);
        collected++;
    }
    return reward;
}

// ---------------------------------------------------------------------------------------------
// One environment of a batch (batch_core.h).

enum { kObsSimple115 = 1, kObsSimple115v2 = 2, kObsSmm = 4, kObsRaw = 8 };
constexpr int kSimple115 = 115;
// GRF's super mini map ("extracted"): kSmmLayers channels per cell (left team, right team, ball,
// active player), 255 at marked cells and 0 elsewhere.
constexpr int kSmmLayers = 4;
constexpr int kSmmMarks = 2 * kTeamPlayers + 2;  // every player, the ball, the active player
constexpr int kSmmMarkRow = 1 + kSmmMarks;       // a frame's mark count, then its marks
// GRF's raw observation as separate arrays (batch_core.h:53-210): one array per field, each
// [count][agents][dims...], every array starting at a multiple of 256 bytes of one buffer. The
// field order and names are GRF's observation keys, so readers can index by name.
enum RawField {
    kRawBall, kRawBallDirection, kRawBallRotation, kRawBallOwnedTeam, kRawBallOwnedPlayer,
    kRawLeftTeam, kRawLeftTeamDirection, kRawLeftTeamTired, kRawLeftTeamYellow, kRawLeftTeamActive, kRawLeftTeamRoles,
    kRawRightTeam, kRawRightTeamDirection, kRawRightTeamTired, kRawRightTeamYellow, kRawRightTeamActive,
    kRawRightTeamRoles, kRawScore, kRawStepsLeft, kRawGameMode, kRawActive, kRawDesignated, kRawSticky, kRawFields
};
enum RawType { kRawF32 = 0, kRawI32 = 1, kRawBool = 2, kRawU8 = 3 };
struct RawArray {
    int32_t type, dims[2], elements;  // dims after the agent axis, 0 when absent
    uint64_t offset;                  // bytes into the raw buffer
};
struct RawLayout {
    int32_t players;  // each team array's length: the larger team of any bundle
    RawArray arrays[kRawFields];
    uint64_t bytes;
};

// Per-environment books (batch_core.h:343 EnvironmentSlot).
struct EnvSlot {
    EpisodeGen gen;
    int32_t episode;  // resets so far
    int32_t reverse;  // the run's team order
    uint32_t seed;
    int32_t variant;  // bundle * 4 + reverse * 2 + parity
    int32_t bundle;
    int32_t leftAgents, rightAgents;
    int32_t collected[kAgentsMax];
    uint8_t sticky[kAgentsMax][kMaxSticky];
    int64_t fixedSeed;      // GRF game_engine_random_seed, or -1 to draw
    int32_t episodeOffset;  // GRF episode_number
    int32_t finalDesignated[2];
};

// Per-variant read-only data: the template match and its context, in device memory.
struct Variant {
    const Match *tmpl;
    Context ctx;
};

// The batch buffers (batch_core.h:368 EnvironmentBuffers), in device memory.
struct Batch {
    Match *worlds;
    EnvCore *cores;
    EnvSlot *slots;
    WarpScratch *scratch;  // one per environment
    int32_t *status;       // one per environment; 0 while every call succeeded
    int32_t *anyFail;      // the first failure code of any environment, 0 for none
    const Variant *variants;
    int agents, count;
    int actionSet, observation;
    bool checkpoints, numpyLegacy, autoReset;
    int stack;
    float *simple115, *finalSimple115;  // [count][agents][115 * stack], null without simple115
    uint8_t *smm, *finalSmm;            // [count][agents][smmHeight][smmWidth][4 * stack], or null
    int32_t *smmMarks, *finalSmmMarks;  // [count][agents][stack][kSmmMarkRow]: each frame's marks
    int smmWidth, smmHeight;
    uint8_t *raw, *finalRaw;            // the raw arrays of `rawLayout`, or null
    RawLayout rawLayout;
    float *reward;                      // [count][agents]
    uint8_t *done;                      // [count]
    int32_t *scoreReward;               // [count]
    const float *teamDifficulty;        // [count][2], negative for the scenario's, or null
    int crewLog2;                       // log2 of the lanes that run each environment (0 to 5)
};

CB_HD int variant_of(const EnvSlot &s) { return s.bundle * 4 + s.reverse * 2 + ((s.episode - 1 + s.episodeOffset) & 1); }

CB_HDNI void update_sticky(const Batch &b, Match &w, EnvSlot &slot) {
    for (int a = 0; a < slot.leftAgents + slot.rightAgents; a++) {
        const bool left = a < slot.leftAgents;
        const int c = sticky_count(b.actionSet);
        for (int i = 0; i < c; i++)
            slot.sticky[a][i] = sticky_action_state(w, sticky_action(i), left, left ? a : a - slot.leftAgents);
    }
}

// The per-environment state a call works on.
CB_HD Sim make_sim(const Batch &b, int e, const Context &ctx) {
    return Sim{b.worlds[e], ctx, b.scratch + e, b.status + e};
}

/// batch_core.h:262 (ResetEnvironment). Each scenario GRF builds draws randint(0, 2e9); creating
/// an environment builds three (two configurations, then the core's reset) and the second's parity
/// sets the run's team order. A given seed, or a fixed one, replaces every draw.
CB_HDNI bool reset_environment(const Batch &b, int e, const int64_t *seeds, const int32_t *reverse) {
    EnvSlot &slot = b.slots[e];
    // Lane 0 keeps the books; the other lanes read them after the barrier.
    crew_sync();
    if (leader()) {
        const bool given = seeds && seeds[e] >= 0;
        const bool fixed = slot.fixedSeed >= 0;
        const bool deterministic = b.variants[slot.bundle * 4].tmpl->scenario.deterministic;
        if (slot.episode == 0) {
            uint32_t creation[3];
            for (int d = 0; d < 3; d++)
                creation[d] = given ? (uint32_t)seeds[e] : fixed ? (uint32_t)slot.fixedSeed : episode_draw_seed(slot.gen);
            slot.reverse = reverse ? reverse[e] : deterministic ? 0 : (int32_t)(creation[1] & 1);
        }
        slot.seed = given ? (uint32_t)seeds[e] : fixed ? (uint32_t)slot.fixedSeed : episode_draw_seed(slot.gen);
        slot.episode++;
        slot.variant = variant_of(slot);
        if (deterministic) slot.seed = b.variants[slot.variant].tmpl->scenario.gameEngineRandomSeed;
    }
    crew_sync();
    struct {
        int32_t variant;
        uint32_t seed;
    } sl = {slot.variant, slot.seed};
    const Variant &v = b.variants[sl.variant];
    Match &w = b.worlds[e];
    crew_copy(w, *v.tmpl);
    // The difficulty goes in before the ticks that bring the match into play, which read it.
    if (b.teamDifficulty) {
        const float l = b.teamDifficulty[e * 2], r = b.teamDifficulty[e * 2 + 1];
        if (l >= 0.0f) w.scenario.leftTeamDifficulty = l;
        if (r >= 0.0f) w.scenario.rightTeamDifficulty = r;
    }
    crew_sync();
    Sim s = make_sim(b, e, v.ctx);
    if (!reset_from_template(s, sl.seed) || !core_after_reset(s, b.cores[e])) return false;
    crew_sync();
    for (int a = 0; a < kAgentsMax; a++) slot.collected[a] = 0;
    update_sticky(b, w, slot);
    crew_sync();
    return true;
}

/// observation_encoding.h:124 (SmmIndex): the byte of `layer` at the cell of a position in the
/// observation's coordinates (x in [-1, 1], y in [-1/2.25, 1/2.25]), truncated toward zero in
/// double and clamped into the map.
CB_HD int smm_cell(int layer, double x, double y, int width, int height) {
    const double x0 = -1.0, x1 = 1.0, y0 = -1.0 / 2.25, y1 = 1.0 / 2.25;
    int col = cvt_d_i32((x - x0) / (x1 - x0) * width);
    int row = cvt_d_i32((y - y0) / (y1 - y0) * height);
    col = col < 0 ? 0 : (col > width - 1 ? width - 1 : col);
    row = row < 0 ? 0 : (row > height - 1 ? height - 1 : row);
    return (row * width + col) * kSmmLayers + layer;
}
/// observation_encoding.h:135 (SmmMarks): the marked bytes of one frame, in GRF's drawing order.
CB_HD int smm_frame_marks(const AgentView &v, int32_t *marks, int width, int height) {
    int n = 0;
    for (int t = 0; t < 2; t++)
        for (int p = 0; p < v.o.team[t].count; p++)
            marks[n++] = smm_cell(t, v.o.team[t].players[p].position[0], v.o.team[t].players[p].position[1], width,
                                  height);
    marks[n++] = smm_cell(2, v.o.ball[0], v.o.ball[1], width, height);
    if (v.active != -1)
        marks[n++] = smm_cell(3, v.o.team[0].players[v.active].position[0],
                              v.o.team[0].players[v.active].position[1], width, height);
    return n;
}
// Sets (or clears) every marked byte of a stacked map: frame f of the stack sits at channels
// [4 f, 4 f + 4) of each cell, and a mark names a byte of one frame.
CB_HD void smm_paint(uint8_t *map, const int32_t *marks, int stack, uint8_t value) {
    const int channels = kSmmLayers * stack;
    for (int f = 0; f < stack; f++) {
        const int32_t *row = marks + f * kSmmMarkRow;
        for (int k = 0; k < row[0]; k++) {
            const int m = row[1 + k];
            map[(size_t)(m / kSmmLayers) * channels + kSmmLayers * f + m % kSmmLayers] = value;
        }
    }
}
/// batch_core.h:534 (the SMM part of WriteAgentOutputs). A map is zero but for its marks, so a
/// write clears the previous marks, moves the frames one place toward the oldest (a reset fills
/// every frame with the new one), and paints the marks again; the final map of an ended episode
/// copies the same way.
CB_HDNI void write_agent_smm(const Batch &b, size_t out, const AgentView &v, bool afterStep, bool finished) {
    const int stack = b.stack;
    const size_t mapBytes = (size_t)b.smmWidth * b.smmHeight * kSmmLayers * stack;
    uint8_t *map = b.smm + out * mapBytes;
    int32_t *marks = b.smmMarks + out * kSmmMarkRow * stack;
    smm_paint(map, marks, stack, 0);
    if (afterStep)
        for (int i = 0; i < (stack - 1) * kSmmMarkRow; i++) marks[i] = marks[i + kSmmMarkRow];
    int32_t *newest = marks + (stack - 1) * kSmmMarkRow;
    newest[0] = smm_frame_marks(v, newest + 1, b.smmWidth, b.smmHeight);
    if (!afterStep)
        for (int i = 0; i < (stack - 1) * kSmmMarkRow; i++) marks[i] = newest[i % kSmmMarkRow];
    smm_paint(map, marks, stack, 255);
    if (finished) {
        uint8_t *finalMap = b.finalSmm + out * mapBytes;
        int32_t *finalMarks = b.finalSmmMarks + out * kSmmMarkRow * stack;
        smm_paint(finalMap, finalMarks, stack, 0);
        for (int i = 0; i < stack * kSmmMarkRow; i++) finalMarks[i] = marks[i];
        smm_paint(finalMap, finalMarks, stack, 255);
    }
}

/// batch_core.h:162 (WriteRaw): one agent's view into every raw array; team arrays shorter than
/// the layout's players pad with zeros.
CB_HDNI void write_agent_raw(const RawLayout &lay, uint8_t *buf, size_t out, const AgentView &v, int stepsLeft) {
    auto at = [&](int field, int index) {
        const RawArray &a = lay.arrays[field];
        const int size = a.type == kRawF32 || a.type == kRawI32 ? 4 : 1;
        return buf + a.offset + ((size_t)out * a.elements + index) * size;
    };
    auto f32 = [&](int field, int index, float x) { memcpy(at(field, index), &x, 4); };
    auto i32 = [&](int field, int index, int32_t x) { memcpy(at(field, index), &x, 4); };
    auto u8 = [&](int field, int index, int x) { *at(field, index) = (uint8_t)x; };
    const Observation &o = v.o;
    for (int k = 0; k < 3; k++) {
        f32(kRawBall, k, o.ball[k]);
        f32(kRawBallDirection, k, o.ballDirection[k]);
        f32(kRawBallRotation, k, o.ballRotation[k]);
    }
    i32(kRawBallOwnedTeam, 0, o.ballOwnedTeam);
    i32(kRawBallOwnedPlayer, 0, o.ballOwnedPlayer);
    for (int t = 0; t < 2; t++) {
        const TeamObs &team = o.team[t];
        const int base = t == 0 ? kRawLeftTeam : kRawRightTeam;
        for (int p = 0; p < lay.players; p++) {
            const bool here = p < team.count;
            const PlayerObs &po = team.players[here ? p : 0];
            for (int c = 0; c < 2; c++) {
                f32(base, 2 * p + c, here ? po.position[c] : 0.0f);
                f32(base + 1, 2 * p + c, here ? po.direction[c] : 0.0f);
            }
            f32(base + 2, p, here ? po.tiredFactor : 0.0f);
            u8(base + 3, p, here && po.yellowCard);
            u8(base + 4, p, here && po.active);
            i32(base + 5, p, here ? po.role : 0);
        }
    }
    i32(kRawScore, 0, o.score[0]);
    i32(kRawScore, 1, o.score[1]);
    i32(kRawStepsLeft, 0, stepsLeft);
    i32(kRawGameMode, 0, o.gameMode);
    i32(kRawActive, 0, v.active);
    i32(kRawDesignated, 0, v.designated);
    for (int i = 0; i < lay.arrays[kRawSticky].elements; i++) u8(kRawSticky, i, i < v.stickyCount ? v.sticky[i] : 0);
}

/// batch_core.h:366 (WriteAgentOutputs) for simple115: one lane, one agent. A step that ends an
/// episode also writes final_simple115.
CB_HDNI void write_agent_outputs(const Batch &b, int e, int agent, bool afterStep) {
    const size_t out = (size_t)e * b.agents + agent;
    EnvSlot &slot = b.slots[e];
    const bool right = agent >= slot.leftAgents;
    AgentView v;
    make_agent_view(b.cores[e].observation, right, right ? agent - slot.leftAgents : agent, b.actionSet,
                    slot.sticky[agent], v);
    if (afterStep && b.checkpoints)
        b.reward[out] = checkpoint_reward(v, b.reward[out], slot.collected[agent], b.numpyLegacy);
    const bool finished = afterStep && b.done[e];
    const int stack = b.stack;
    if (b.observation & (kObsSimple115 | kObsSimple115v2)) {
        const int width = kSimple115 * stack;
        float *st = b.simple115 + out * width;
        float *enc = st + width - kSimple115;
        // As FrameStack: the last `stack` observations, oldest first; a reset fills every frame.
        if (afterStep)
            for (int i = 0; i < width - kSimple115; i++) st[i] = st[i + kSimple115];
        encode_simple115(v, (b.observation & kObsSimple115v2) != 0, enc);
        if (!afterStep)
            for (int i = 0; i < width - kSimple115; i++) st[i] = enc[i % kSimple115];
        if (finished)
            for (int i = 0; i < width; i++) b.finalSimple115[out * width + i] = st[i];
    }
    if (b.observation & kObsSmm) write_agent_smm(b, out, v, afterStep, finished);
    if (b.observation & kObsRaw) {
        const int stepsLeft = b.worlds[e].scenario.gameDuration - v.o.step;
        write_agent_raw(b.rawLayout, b.raw, out, v, stepsLeft);
        if (finished) write_agent_raw(b.rawLayout, b.finalRaw, out, v, stepsLeft);
    }
}

// One agent per lane.
CB_HDNI void write_env_outputs(const Batch &b, int e, bool afterStep) {
    crew_sync();
    const EnvSlot &slot = b.slots[e];
    const int n = slot.leftAgents + slot.rightAgents;
    crew_for(n, [&](int a) { write_agent_outputs(b, e, a, afterStep); });
    crew_sync();
}

// An iteration cap of GRF's arithmetic reached during a call (crew_note_cap) marks a path GRF
// leaves undefined: the environment's status says so, and the host raises it at the next
// synchronising call.
CB_HD void settle_caps(const Batch &b, int e) {
    if (crew_cap_reached() && b.status[e] == kStatusOk) b.status[e] = kStatusUnsupported;
    crew_clear_cap();
}

CB_HDNI bool reset_and_write(const Batch &b, int e, const int64_t *seeds, const int32_t *reverse) {
    if (!reset_environment(b, e, seeds, reverse)) return false;
    if (leader()) b.done[e] = 0;
    write_env_outputs(b, e, false);
    return true;
}

/// batch_core.h:601 (StepEnvironment). With autoReset an ended episode resets in the same call,
/// done still set; without it the environment keeps its outputs until a reset. Actions out of
/// range act as idle; a negative index counts from the end of the action list.
CB_HDNI bool step_environment(const Batch &b, int e, const int32_t *actions) {
    EnvSlot &slot = b.slots[e];
    const int agents = slot.leftAgents + slot.rightAgents;
    if (!b.autoReset && b.done[e]) {
        crew_sync();
        if (leader()) {
            for (int a = 0; a < b.agents; a++) b.reward[(size_t)e * b.agents + a] = 0.0f;
            b.scoreReward[e] = 0;
        }
        return true;
    }
    int ea[kAgentsMax];
    for (int a = 0; a < agents; a++) {
        const bool right = a >= slot.leftAgents;
        int ix = actions[(size_t)e * b.agents + a];
        const int n = action_set_size(b.actionSet);
        if (ix < 0) ix += n;
        if (ix < 0 || ix >= n) ix = 0;
        // A right agent acts on the flipped pitch: its direction turns back by both axes.
        ea[a] = negate_action_axes(action_from_set(ix), right, right);
    }
    int reward = 0;
    bool done = false;
    Match &w = b.worlds[e];
    Sim s = make_sim(b, e, b.variants[slot.variant].ctx);
    if (!core_step(s, b.cores[e], ea, reward, done)) return false;
    crew_sync();
    update_sticky(b, w, slot);
    crew_sync();
    if (leader()) {
        for (int a = 0; a < b.agents; a++)
            b.reward[(size_t)e * b.agents + a] = a < agents ? (float)(a < slot.leftAgents ? reward : -reward) : 0.0f;
        b.done[e] = done;
        b.scoreReward[e] = reward;
    }
    write_env_outputs(b, e, true);
    if (done && leader())
        for (int t = 0; t < 2; t++) slot.finalDesignated[t] = b.cores[e].observation.team[t].designatedPlayer;
    crew_sync();
    if (!b.autoReset || !done) return true;
    if (!reset_environment(b, e, nullptr, nullptr)) return false;
    write_env_outputs(b, e, false);
    return true;
}

}  // namespace cb
