// cuju-b200: per-match accessors and the small per-player helpers every subsystem reads.
//   frames / mirroring      cuju include/cuju/simulation/world.h:52-167
//   team & humanoid access  cuju include/cuju/simulation/access.h:14-62
//   spatial state           cuju include/cuju/simulation/humanoid.h:108-419
//   possession statistics   cuju include/cuju/simulation/player_possession.h:17-123
//   pass / shot direction   cuju include/cuju/simulation/ai_functions.h:15-187
//   keyboard input          cuju include/cuju/simulation/human_controller.h:12-114
#pragma once

#include "ball.cuh"
#include "tables.cuh"
#include "assist.cuh"

namespace cb {

enum Velocity { kVelIdle, kVelDribble, kVelWalk, kVelSprint };
enum FunctionType {
    kFtNone, kFtMovement, kFtBallControl, kFtTrap, kFtShortPass, kFtLongPass, kFtHighPass,
    kFtHeader, kFtShot, kFtDeflect, kFtCatch, kFtInterfere, kFtTrip, kFtSliding, kFtSpecial
};
enum TouchType { kTouchKicked, kTouchNonKicked, kTouchAccidental, kTouchNone };
enum Role {
    kRoleGK, kRoleCB, kRoleLB, kRoleRB, kRoleDM, kRoleCM, kRoleLM, kRoleRM, kRoleAM, kRoleCF
};
enum GameMode { kGmNormal, kGmKickOff, kGmGoalKick, kGmFreeKick, kGmCorner, kGmThrowIn, kGmPenalty };
enum Strict { kStrictFalse, kStrictTrue, kStrictDynamic };
enum BodyPart {
    kBpMiddle, kBpNeck, kBpLeftThigh, kBpRightThigh, kBpLeftKnee, kBpRightKnee, kBpLeftAnkle,
    kBpRightAnkle, kBpLeftShoulder, kBpRightShoulder, kBpLeftElbow, kBpRightElbow, kBpBody,
    kBpPlayer
};
enum Interrupt {
    kIntNone, kIntSwitch, kIntSliding, kIntBump, kIntTrip, kIntCheat, kIntCancel, kIntReQueue
};
enum MatchPhase { kPhasePreMatch, kPhaseFirstHalf, kPhaseSecondHalf };
enum Button {
    kBtnLongPass, kBtnHighPass, kBtnShortPass, kBtnShot, kBtnKeeperRush, kBtnSliding,
    kBtnPressure, kBtnTeamPressure, kBtnSwitch, kBtnSprint, kBtnDribble, kBtnCount
};
constexpr int kFootRight = 1;
constexpr float kStickDeadzone = 0.75f;

// Fixed-capacity scratch lists (not part of the state).
template <class T, int N>
struct List {
    int32_t count = 0;
    T el[N];
    CB_HD void push(const T &v) { el[count++] = v; }
    CB_HD T &operator[](int i) { return el[i]; }
    CB_HD const T &operator[](int i) const { return el[i]; }
    CB_HD void erase_at(int i) {
        for (int k = i; k + 1 < count; k++) el[k] = el[k + 1];
        count--;
    }
};
using PlayerList = List<int, kPlayers>;

// ---------------------------------------------------------------------------------------------
// Teams and humanoids. A team ID is 0/1 (scenario left/right); its slot is its place in
// processing order; teams[0] is the team processed first.
CB_HD int team_slot(const Match &w, int teamID) { return teamID == w.firstTeamID() ? 0 : 1; }
CB_HD Team &team_by_id(Match &w, int teamID) { return w.m.teams[team_slot(w, teamID)]; }
CB_HD const Team &team_by_id(const Match &w, int teamID) { return w.m.teams[team_slot(w, teamID)]; }
CB_HD const Team &team_of(const Match &w, int p) { return team_by_id(w, w.playerTeamID[p]); }
CB_HD const Team &opp_team_of(const Match &w, int p) { return team_by_id(w, 1 - w.playerTeamID[p]); }
CB_HD Humanoid &hum(Match &w, int p) { return w.m.players[p].base.humanoid; }
CB_HD const Humanoid &hum(const Match &w, int p) { return w.m.players[p].base.humanoid; }
// Players first, then the officials.
CB_HD Humanoid &any_hum(Match &w, int h) {
    return h < w.m.playerCount ? w.m.players[h].base.humanoid
                               : w.m.officials[h - w.m.playerCount].humanoid;
}
CB_HD Vec3 ball_at(const Match &w, int t_ms) { return ball_predict(w.m.ball, t_ms); }

CB_HD int gamer_count_enabled(const Team &t) {
    int n = 0;
    for (int g = 0; g < t.gamers.count; g++)
        if (!t.gamers[g].controller.keyboard.disabled) n++;
    return n;
}
CB_HD void init_player_teams(Match &w) {
    int first = w.firstTeamID();
    int firstSize = first == 0 ? w.scenario.leftTeamSize : w.scenario.rightTeamSize;
    for (int p = 0; p < w.m.playerCount; p++) w.playerTeamID[p] = p < firstSize ? first : 1 - first;
    for (int p = 0; p < kPlayers; p++) w.formationOverride[p] = 0;
}
CB_HD int formation_source(const Match &w, int p) {
    const int o = w.formationOverride[p];
    return o ? o - 1 : p;
}
CB_HD const StaticFormation &formation(const Sim &s, int p) {
    return s.ctx.staticData->formation[formation_source(s.w, p)];
}

// ---------------------------------------------------------------------------------------------
// Mirroring: each team is processed in its own frame; a mirror negates x and y exactly.
CB_HDNI void mirror_humanoid(Humanoid &h, bool &mirrored) {
    NodeState &root = h.nodes[0];
    root.position = root.position * Vec3(-1, -1, 1);
    Quat r = root.rotation;
    if (!mirrored)
        root.rotation = Quat(r.e[1], r.e[0], r.e[3], -r.e[2]);
    else
        root.rotation = Quat(r.e[1], r.e[0], -r.e[3], r.e[2]);
    mirrored = !mirrored;
    h.startPosition.mirror();
    h.startAngle.rotated = !h.startAngle.rotated;
    h.nextStartPosition.mirror();
    h.nextStartAngle.rotated = !h.nextStartAngle.rotated;
    SpatialState &s = h.spatial;
    s.position.mirror();
    s.actualMovement.mirror();
    s.physicsMovement.mirror();
    s.animationMovement.mirror();
    s.movement.mirror();
    s.actionSmuggleMovement.mirror();
    s.movementSmuggleMovement.mirror();
    s.positionOffsetMovement.mirror();
    h.previousPosition2D.mirror();
    h.tripDirection.mirror();
    h.decayingPositionOffset.mirror();
}
CB_HD void mirror_team(Match &w, int teamID) {
    w.flags.teamSide[teamID] *= -1;
    w.flags.teamMirrored[teamID] = !w.flags.teamMirrored[teamID];
    crew_for(w.m.playerCount, [&](int p) {
        if (w.playerTeamID[p] == teamID) mirror_humanoid(w.m.players[p].base.humanoid, w.flags.humanoidMirrored[p]);
    });
}
CB_HD void mirror_ball(Ball &b) {
    b.momentum.mirror();
    b.lazyFlip = !b.lazyFlip;
    b.positionBuffer.mirror();
}
// Applies a pending lazy mirror to the whole prediction and history arrays.
CB_HD void ball_materialize(Ball &b) {
    if (!b.lazyFlip) return;
    const int n = 401;
    crew_for(n + b.positionHistory.count, [&](int i) {
        if (i < n) b.predictions[i].mirror();
        else b.positionHistory[i - n].mirror();
    });
    b.lazyFlip = false;
}
CB_HD void mental_materialize(MentalImage &im) {
    if (!im.lazyFlip) return;
    crew_for(im.ballPredictions.count, [&](int i) { im.ballPredictions[i].mirror(); });
    im.lazyFlip = false;
}
CB_HD void mirror_mental(Match &w, int idx, bool t0, bool t1, bool ball) {
    MentalImage &im = w.m.mentalImages[idx];
    crew_for(im.players.count, [&](int i) {
        PlayerImage &pi = im.players[i];
        int team = w.playerTeamID[pi.player];
        if (team == 0 ? t0 : t1) {
            pi.position.mirror();
            pi.directionVector.mirror();
            pi.movement.mirror();
        }
    });
    if (ball) {
        im.lazyFlip = !im.lazyFlip;
        w.flags.mentalBallMirrored[idx] = !w.flags.mentalBallMirrored[idx];
    }
}
CB_HD void mirror_match(Match &w, bool t0, bool t1, bool ball) {
    if (t0) mirror_team(w, 0);
    if (t1) mirror_team(w, 1);
    if (ball) {
        w.flags.ballMirrored = !w.flags.ballMirrored;
        mirror_ball(w.m.ball);
    }
    for (int i = 0; i < w.m.mentalImages.count; i++) mirror_mental(w, i, t0, t1, ball);
}
// The state stores ball, last-touch team IDs and referee buffer relative to processing order;
// an involution.
CB_HDNI void canonical_to_rest(Match &w) {
    MatchState &m = w.m;
    if (w.firstTeamID() == 1) {
        for (int i = 0; i < 4; i++)
            if (m.lastTouchTeamIDs[i] != -1) m.lastTouchTeamIDs[i] = 1 - m.lastTouchTeamIDs[i];
        if (m.lastTouchTeamID != -1) m.lastTouchTeamID = 1 - m.lastTouchTeamID;
    }
    if (!w.scenario.reverseTeamProcessing) return;
    mirror_ball(m.ball);
    for (int i = 0; i < m.mentalImages.count; i++) m.mentalImages[i].lazyFlip = !m.mentalImages[i].lazyFlip;
    m.referee.buffer.teamID = 1 - m.referee.buffer.teamID;
    m.referee.buffer.restartPosition.mirror();
    m.referee.foul.foulPosition.mirror();
}

// ---------------------------------------------------------------------------------------------
// Velocity categories and angles.
CB_HD float fix_angle(float a) { return wrap_range(-kPi, kPi, a + 0.5f * kPi); }
CB_HD float range_velocity(float v) {
    float r = kIdleVel;
    if (v >= kIdleDribbleSwitch && v < kDribbleWalkSwitch) r = kDribbleVel;
    else if (v >= kDribbleWalkSwitch && v < kWalkSprintSwitch) r = kWalkVel;
    else if (v >= kWalkSprintSwitch) r = kSprintVel;
    return r;
}
CB_HD int vel_category(float v) {
    float r = range_velocity(v);
    if (r == kIdleVel) return kVelIdle;
    if (r == kDribbleVel) return kVelDribble;
    if (r == kWalkVel) return kVelWalk;
    if (r == kSprintVel) return kVelSprint;
    return kVelIdle;
}
CB_HD float vel_float(int c) {
    switch (c) {
        case kVelIdle: return kIdleVel;
        case kVelDribble: return kDribbleVel;
        case kVelWalk: return kWalkVel;
        case kVelSprint: return kSprintVel;
    }
    return 0;
}
CB_HD float player_float_velocity(const Match &w, int p) { return vel_float(hum(w, p).spatial.velocityCategory); }

// The five body directions relative to movement (+ the zero vector at index 5); each angle is a
// multiple of pi computed in double and rounded.
CB_HD Vec3 allowed_body_dir(int i) {
    const float h = 0x1.6a09e6p-1f;
    switch (i) {
        case 0: return Vec3(0.0f, -1.0f, 0.0f);
        case 1: return Vec3(-h, -h, 0.0f);
        case 2: return Vec3(h, -h, 0.0f);
        case 3: return Vec3(-h, h, 0.0f);
        case 4: return Vec3(h, h, 0.0f);
        default: return Vec3(0.0f, 0.0f, 0.0f);
    }
}
// allowed_body_dir(i).angle2d_to(0,-1,0): the first is -0, the last +0.
CB_HD float allowed_body_angle(int i) {
    switch (i) {
        case 0: return -0.0f;
        case 1: return -0x1.921fb6p-1f;
        case 2: return 0x1.921fb6p-1f;
        case 3: return -0x1.2d97c8p+1f;
        case 4: return 0x1.2d97c8p+1f;
        default: return 0.0f;
    }
}
// Index of the allowed direction with the largest dot product above -1; 5 if none.
CB_HDNI int force_allowed_body_index(const Vec3 &v) {
    float best = -1.0f;
    int bi = 5;
    for (int i = 0; i < 5; i++) {
        float d = allowed_body_dir(i).dot(v);
        if (d > best) {
            best = d;
            bi = i;
        }
    }
    return bi;
}
CB_HD Vec3 force_allowed_body_vector(const Vec3 &v) { return allowed_body_dir(force_allowed_body_index(v)); }

// Movement (m/s, ground plane) at a frame of a position list of two frames or more.
template <class P>
CB_HDNI Vec3 movement_at_frame(const P &pos, int count, uint32_t frame, uint32_t smooth) {
    if (frame == (uint32_t)(count - 1)) return (pos[count - 1] - pos[count - 2]).flat() * 100.0f;
    if (frame == 0) return (pos[1] - pos[0]).flat() * 100.0f;
    Vec3 total;
    uint32_t n = 0;
    for (int f = (int)(frame - smooth); f <= (int)(frame + smooth); f++) {
        if (f > 0 && f < count) {
            total += (pos[f] - pos[f - 1]).flat() * 100.0f;
            n++;
        }
    }
    if (n > 0) total /= Vec3((float)n);
    return total;
}

// ---------------------------------------------------------------------------------------------
// Animation keyframes (cuju include/cuju/animation/keyframes.h:16-91).
CB_HDNI void interpolate_keys(const Anim &a, const KeyFrame *keys, int nkeys, int frame, Quat &o,
                              Vec3 &p) {
    struct WK {
        const KeyFrame *k;
        float infl;
        int frame;
    } wk[2] = {{nullptr, 0.0f, 0}, {nullptr, 0.0f, 0}};
    int n = 0;
    p = Vec3(0);
    o = Quat::identity();
    if (frame > 0 && frame < a.frameCount) {
        for (int k = 0; k < nkeys; k++) {
            if (keys[k].frame < frame) n = 0;
            wk[n].k = &keys[k];
            wk[n++].frame = keys[k].frame;
            if (keys[k].frame >= frame) break;
        }
        float bias = 0;
        if (n == 1) {
            wk[0].infl = 1;
        } else if (n == 2) {
            int dist = wk[1].frame - wk[0].frame;
            float d1 = frame - wk[0].frame;
            float d2 = wk[1].frame - frame;
            wk[0].infl = (float)(1 - d1 / (dist * 1.0));
            wk[1].infl = (float)(1 - d2 / (dist * 1.0));
            int rel = frame - wk[0].frame;
            bias = (float)((rel * 1.0) / (dist * 1.0));
        }
        if (n > 1) {
            o = wk[0].k->orientation.slerp(bias, wk[1].k->orientation);
            p = wk[0].k->position * wk[0].infl + wk[1].k->position * wk[1].infl;
        } else {
            o = wk[0].k->orientation;
            p = wk[0].k->position * wk[0].infl;
        }
    } else if (frame >= a.frameCount) {
        for (int k = nkeys; k-- > 0;) {
            wk[n].k = &keys[k];
            wk[n++].frame = keys[k].frame;
            if (n == 2) break;
        }
        if (n == 0) return;
        if (n == 1) {
            o = wk[0].k->orientation;
            p = wk[0].k->position;
            return;
        }
        float spacing = wk[0].frame - wk[1].frame;
        float past = frame - wk[0].frame;
        float bias = 1 + ((1 / spacing) * past);
        o = wk[1].k->orientation.slerp(bias, wk[0].k->orientation);
        p = wk[1].k->position * (1 - bias) + wk[0].k->position * bias;
    } else {
        o = keys[0].orientation;
        p = keys[0].position;
    }
}
CB_HD void node_pose(const AnimTables &T, const Anim &a, const NodeAnim &n, int frame, Quat &o,
                     Vec3 &p) {
    if (n.interpFrames > 0 && frame < n.interpFrames) {
        const InterpEntry &e = T.interp[n.interpOffset + (frame < 0 ? 0 : frame)];
        o = e.orientation;
        p = e.position;
        return;
    }
    interpolate_keys(a, T.keys + n.firstKey, n.keyCount, frame, o, p);
}
CB_HD void node_pose_z(const AnimTables &T, const Anim &a, const NodeAnim &n, int frame, Quat &o,
                       Vec3 &p, float &z) {
    if (n.interpFrames > 0 && frame < n.interpFrames) {
        const InterpEntry &e = T.interp[n.interpOffset + (frame < 0 ? 0 : frame)];
        o = e.orientation;
        p = e.position;
        z = e.angleZ;
        return;
    }
    interpolate_keys(a, T.keys + n.firstKey, n.keyCount, frame, o, p);
    float x, y;
    o.angles(x, y, z);
}
// The yaw of a body part at a frame; the angles of the (unset) identity if the animation has no
// such node.
CB_HD void key_frame_z(const AnimTables &T, const Anim &a, int bodyPart, int frame, Quat &o, Vec3 &p,
                       float &z) {
    for (int i = 0; i < a.nodeCount; i++) {
        const NodeAnim &n = T.nodes[a.firstNode + i];
        if (n.bodyPart == bodyPart) {
            node_pose_z(T, a, n, frame, o, p, z);
            return;
        }
    }
    float x, y;
    o.angles(x, y, z);
}
CB_HD bool key_frame(const AnimTables &T, const Anim &a, int bodyPart, int frame, Quat &o, Vec3 &p) {
    for (int i = 0; i < a.nodeCount; i++) {
        const NodeAnim &n = T.nodes[a.firstNode + i];
        if (n.bodyPart == bodyPart) {
            node_pose(T, a, n, frame, o, p);
            for (int k = 0; k < n.keyCount; k++)
                if (T.keys[n.firstKey + k].frame == frame) return true;
            return false;
        }
    }
    return false;
}

// ---------------------------------------------------------------------------------------------
// Spatial state of a humanoid after its animation frame advanced (GRF Humanoid::CalculateSpatialState).
CB_HDNI void calc_spatial_state(const Sim &s, Humanoid &h) {
    AnimationState &ca = h.anim;
    const Anim &a = s.A(ca.anim);
    SpatialState &sp = h.spatial;
    Vec3 position;
    if ((uint32_t)ca.positions.count > (uint32_t)ca.frameNumber) {
        position = h.startPosition + ca.positions[ca.frameNumber] + ca.actionSmuggleOffset +
                   ca.actionSmuggleSustainOffset + ca.movementSmuggleOffset;
    } else {
        Quat o;
        key_frame(s.T(), a, kBpPlayer, ca.frameNumber, o, position);
        position.c[2] = 0.0f;
        position = h.startPosition + rot2d(position, h.startAngle.value()) + ca.actionSmuggleOffset +
                   ca.actionSmuggleSustainOffset + ca.movementSmuggleOffset;
    }
    if (ca.frameNumber > 12) sp.foot = a.outgoingFoot;
    sp.actualMovement = (position - h.previousPosition2D) * 100.0f;
    const float ignore = 0.5f;
    sp.physicsMovement = sp.actualMovement - (sp.actionSmuggleMovement) - (sp.movementSmuggleMovement) -
                         (sp.positionOffsetMovement * ignore);
    sp.animationMovement = sp.physicsMovement;
    if (ca.positions.count > 0) {
        sp.animationMovement =
            rot2d(movement_at_frame(s.T().positions + a.firstPosition, a.positionCount, ca.frameNumber, 1),
                  h.startAngle.value());
    }
    sp.movement = sp.physicsMovement;
    Vec3 bodyPos;
    Quat bodyRot;
    float z;
    key_frame_z(s.T(), a, kBpBody, ca.frameNumber, bodyRot, bodyPos, z);
    Vec3 bodyDir = rot2d(Vec3(0, -1, 0), z + h.startAngle.value() + ca.rotationSmuggleOffset.value());
    sp.floatVelocity = sp.movement.length();
    sp.velocityCategory = vel_category(sp.floatVelocity);
    if (sp.velocityCategory != kVelIdle)
        sp.directionVector = sp.movement.normalized();
    else
        sp.directionVector = bodyDir;
    sp.position = position;
    set_radian(sp.angle, wrap_range(-kPi, kPi, fix_angle(angle2d(sp.directionVector))));
    int bodyIdx = 0;
    float nonQuantized = allowed_body_angle(0);
    if (sp.velocityCategory != kVelIdle) {
        Vec3 adapted = rot2d(bodyDir, -sp.angle.value());
        float rel = angle2d_to(adapted, Vec3(0, -1, 0));
        nonQuantized = rel;
        if (sp.velocityCategory == kVelSprint && fabsf(rel) >= 0.125f * kPi) {
            adapted = rot2d(Vec3(0, -1, 0), 0.12f * kPi * sign_side(rel));
            nonQuantized = angle2d_to(adapted, Vec3(0, -1, 0));
        } else if (sp.velocityCategory == kVelWalk && fabsf(rel) >= 0.5f * kPi) {
            adapted = rot2d(Vec3(0, -1, 0), 0.495f * kPi * sign_side(rel));
            nonQuantized = angle2d_to(adapted, Vec3(0, -1, 0));
        }
        sp.relBodyDirectionVectorNonQuantized = adapted;
        bodyIdx = force_allowed_body_index(adapted);
    } else {
        sp.relBodyDirectionVectorNonQuantized = Vec3(0, -1, 0);
    }
    sp.relBodyDirectionVector = allowed_body_dir(bodyIdx);
    set_radian(sp.relBodyAngle, allowed_body_angle(bodyIdx));
    set_radian(sp.relBodyAngleNonQuantized, nonQuantized);
    sp.bodyDirectionVector = rot2d(sp.relBodyDirectionVector, sp.angle.value());
    set_radian(sp.bodyAngle, angle2d_to(sp.bodyDirectionVector, Vec3(0, -1, 0)));
    h.previousPosition2D = position;
}

// std::min operand order: a NaN second operand gives `first`.
CB_HD float std_min(float first, float second) { return (second < first) ? second : first; }
// std::max(left, right): `left` wins a tie or NaN.
CB_HD float std_max(float left, float right) { return (left < right) ? right : left; }

CB_HD float team_difficulty(const Match &w, int teamID) {
    return teamID == 0 ? w.scenario.leftTeamDifficulty : w.scenario.rightTeamDifficulty;
}
CB_HD float statistic(const Sim &s, int p, int st) {
    float mul = 0.3f + 0.7f * team_difficulty(s.w, s.w.playerTeamID[p]);
    mul *= 0.7f + 0.3f * s.w.m.players[p].base.fatigueFactorInverse;
    return s.ctx.staticData->data[p].statistics[st] * mul;
}
CB_HD bool external_active(const Match &w, int p) {
    int ec = w.m.players[p].base.externalController;
    if (ec < 0) return false;
    int first = w.m.teams[0].gamers.count;
    const HumanGamer &g = ec < first ? w.m.teams[0].gamers[ec] : w.m.teams[1].gamers[ec - first];
    return !g.controller.keyboard.disabled;
}
CB_HD int reaction_time_ms(const Sim &s, int p) {
    int rt = cvt_f_i32(roundf(80.0f - statistic(s, p, kStPhysicalReaction) * 40.0f));
    if (external_active(s.w, p)) return rt;
    return cvt_f_i32((float)rt + (1.0f - team_difficulty(s.w, s.w.playerTeamID[p])) * 100);
}
CB_HD float last_touch_bias(const Match &w, int p, int decay_ms) {
    uint64_t t = w.m.actualTime_ms;
    if (decay_ms > 0)
        return 1.0f - clampf_((float)(t - w.m.players[p].base.lastTouchTime_ms) / (float)decay_ms, 0.0f, 1.0f);
    return 0.0f;
}
CB_HD float team_last_touch_bias(const Match &w, int teamID, int decay_ms) {
    int ltp = team_by_id(w, teamID).lastTouchPlayer;
    return ltp >= 0 ? last_touch_bias(w, ltp, decay_ms) : 0.0f;
}
CB_HD void offset_position(Match &w, int p, const Vec3 &off) {
    Humanoid &h = w.m.players[p].base.humanoid;
    h.nextStartPosition += off;
    h.startPosition += off;
    h.spatial.position += off;
    h.spatial.positionOffsetMovement += off * 100.0f;
    h.decayingPositionOffset += off;
    if (h.decayingPositionOffset.length() > 0.1f)
        h.decayingPositionOffset = h.decayingPositionOffset.normalized() * 0.1f;
    h.anim.positionOffset += off;
}
CB_HD int mental_index(const Match &w, int history_ms) {
    int i = cvt_d_i32(round((double)((float)history_ms / 100.0)));
    if (i >= w.m.mentalImages.count) i = w.m.mentalImages.count - 1;
    if (i < 0) i = 0;
    return i;
}
CB_HD Vec3 mental_ball(const Match &w, int imageIdx, int t_ms) {
    const MentalImage &im = w.m.mentalImages[imageIdx];
    // The offset from the image stamp wraps as unsigned 32-bit; outside the window reads the last.
    int i = (int)(uint32_t)((uint64_t)(int64_t)t_ms + w.m.actualTime_ms - (uint64_t)im.timeStamp_ms);
    if ((uint32_t)i >= kPredictionSpan_ms) i = kPredictionSpan_ms - 10;
    i = i / 10;
    if (i < 0) i = 0;
    Vec3 mr = im.ballPredictions[i];
    if (im.lazyFlip) mr.mirror();
    Vec3 rr = ball_at(w, t_ms);
    return mr.max_deviation(rr, im.maxDistanceDeviation);
}

// ---------------------------------------------------------------------------------------------
// Possession (GRF Player::UpdatePossessionStats).
CB_HD float max_velocity(const StaticData &sd, int p) {
    return kSprintVel * (0.9f + sd.data[p].velocityStatistic * 0.1f);
}
CB_HDNI bool has_possession(const Match &w, int p) {
    const Ball &b = w.m.ball;
    const SpatialState &sp = hum(w, p).spatial;
    Vec3 pm = sp.movement;
    if ((double)(sp.position - ball_predict(b, 0)).length() > 5.0) return false;
    if ((double)fabsf(ball_predict(b, 0).c[2]) > 0.5) return false;
    bool dist = true;
    float radius = 1.0f;
    Vec3 center = sp.position + sp.movement * 0.05f + sp.directionVector * 0.1f;
    if ((ball_predict(b, 0).flat() - center).length() > radius) dist = false;
    bool mov = true;
    Vec3 bm = (ball_predict(b, 10) - ball_predict(b, 0)) * 100.0f;
    if ((bm - pm).length() > 6.0f) mov = false;
    return dist && mov;
}
CB_HD bool is_pass_or_shot(int ft) {
    return ft == kFtShortPass || ft == kFtLongPass || ft == kFtHighPass || ft == kFtShot;
}
// Runs on one lane (inside a region): touches only player p.
CB_HDNI void update_possession_stats(Match &w, const StaticData &sd, int p) {
    Player &pl = w.m.players[p];
    const Humanoid &h = pl.base.humanoid;
    const Ball &b = w.m.ball;
    const Team &team = team_of(w, p);
    const Team &opp = opp_team_of(w, p);
    const Vec3 pos = h.spatial.position, mov = h.spatial.movement;
    const float mv = max_velocity(sd, p);
    pl.timeNeededToGetToBallPrevious_ms = pl.timeNeededToGetToBall_ms;
    uint32_t start = 0;
    const bool pending = h.anim.frameNumber < h.anim.touchFrame;
    if (is_pass_or_shot(h.anim.functionType) && !pending) start = 500;
    bool precise = team.designatedTeamPossessionPlayer == p;
    TimeNeeded sc = possession_scan(b.predictions, b.lazyFlip, pos, mov, mv, precise, start);
    pl.timeNeededToGetToBall_ms = sc.usual_ms;
    pl.timeNeededToGetToBallOptimistic_ms = sc.optimistic_ms;
    const bool touchAnim = h.anim.touchFrame != -1;
    if (touchAnim && pending) {
        uint32_t at = (uint32_t)((h.anim.touchFrame - h.anim.frameNumber) * 10);
        if (at < pl.timeNeededToGetToBall_ms) pl.timeNeededToGetToBall_ms = at;
        pl.timeNeededToGetToBallOptimistic_ms = pl.timeNeededToGetToBall_ms;
    }
    if (pl.timeNeededToGetToBall_ms < kTouchOffset_ms) {
        pl.timeNeededToGetToBall_ms = cvt_f_u32(
            nclamp(((pos + mov * (float)(kTouchOffset_ms * 0.001)) - ball_predict(b, kTouchOffset_ms).flat())
                       .length(),
                   0.0f, 0.6f) *
            kTouchOffset_ms);
        pl.timeNeededToGetToBallOptimistic_ms = pl.timeNeededToGetToBall_ms;
    }
    if (is_pass_or_shot(h.anim.functionType) && !pending)
        pl.hasPossession = false;
    else
        pl.hasPossession = has_possession(w, p);
    pl.hasBestPossession =
        pl.hasPossession && opp.timeNeededToGetToBall_ms > (int32_t)pl.timeNeededToGetToBall_ms;
    pl.hasUniquePossession = pl.hasPossession && !opp.hasPossession;
    if (w.m.ballRetainer == p) {
        pl.timeNeededToGetToBall_ms = 1;
        pl.timeNeededToGetToBallOptimistic_ms = 1;
        pl.desiredTimeToBall_ms = (int32_t)pl.timeNeededToGetToBall_ms;
        pl.hasPossession = true;
        pl.hasBestPossession = true;
        pl.hasUniquePossession = true;
    } else if (w.m.ballRetainer != -1) {
        pl.hasPossession = false;
        pl.hasBestPossession = false;
        pl.hasUniquePossession = false;
    }
}

// ---------------------------------------------------------------------------------------------
// Team side, active players, passes and shots.
CB_HD int team_side(const Match &w, int teamID) { return w.flags.teamSide[teamID]; }
// Team rosters go out through a reference: lists returned by value were seen to lose their stack
// slot to later lists of the caller in the sm_100a build.
CB_HD void active_players(PlayerList &l, const Match &w, int teamID) {
    l.count = 0;
    for (int p = 0; p < w.m.playerCount; p++)
        if (w.playerTeamID[p] == teamID && w.m.players[p].base.isActive) l.push(p);
}
CB_HD void all_players(PlayerList &l, const Match &w, int teamID) {
    l.count = 0;
    for (int p = 0; p < w.m.playerCount; p++)
        if (w.playerTeamID[p] == teamID) l.push(p);
}
CB_HD int active_count(const Match &w, int teamID) {
    int n = 0;
    for (int p = 0; p < w.m.playerCount; p++) n += w.playerTeamID[p] == teamID && w.m.players[p].base.isActive;
    return n;
}
CB_HD int team_count(const Match &w, int teamID) {
    int n = 0;
    for (int p = 0; p < w.m.playerCount; p++) n += w.playerTeamID[p] == teamID;
    return n;
}
CB_HDNI void auto_pass(int passType, const Vec3 &v, Vec3 &dir, float &power) {
    float heightOffset = 0.11f, powerFactor = 1.8f, distExp = 1.4f;
    if (passType == kFtHighPass) {
        heightOffset = 0.45f - nclamp(v.length(), 0.0f, 60.0f) * 0.15f;
        powerFactor = 1.15f;
        distExp = 1.4f;
    }
    dir = (v.normalized(Vec3(0)) + Vec3(0, 0, heightOffset)).normalized(Vec3(0));
    power = lm::lm_powf(nclamp(v.length(), 0.0f, 60.0f), distExp) * powerFactor;
}
CB_HDNI void get_pass(const Match &w, int p, int passType, const Vec3 &inputDir, float inputPower,
                      float autoDirBias, float autoPowerBias, Vec3 &outDir, float &outPower,
                      int &targetPlayer, int forcedTarget) {
    const SpatialState &sp = hum(w, p).spatial;
    const AnimationState &ca = hum(w, p).anim;
    const int teamID = w.playerTeamID[p];
    bool fullAutoDir = false, fullAutoPower = false;
    if (external_active(w, p)) {
        fullAutoDir = true;
        fullAutoPower = true;
    }
    float adb = autoDirBias, apb = autoPowerBias;
    Vec3 pp = sp.position + sp.movement.normalized(Vec3(0)) * 0.2f;
    if (ca.touchFrame != -1) pp = ca.touchPosition.flat();
    Vec3 manualTarget = pp + inputDir * clampf_(inputPower * 60.0f, 1.0f, 100.0f);
    PlayerList players;
    active_players(players, w, teamID);
    if (players.count < 2) {
        outDir = sp.directionVector;
        outPower = 1.0f;
        targetPlayer = p;
        fullAutoDir = false;
        fullAutoPower = false;
        adb = 0.0f;
        apb = 0.0f;
    }
    int best = p;
    Vec3 autoTarget = manualTarget;
    if (forcedTarget >= 0) {
        best = forcedTarget;
        const SpatialState &fs = hum(w, forcedTarget).spatial;
        float dur = 0.3f + (fs.position - pp).length() * 0.05f;
        dur = lm::lm_powf(clampf_(dur, 0.0f, 1.0f), 0.7f) * 0.7f;
        autoTarget = fs.position + fs.movement * dur;
    } else {
        float bestRating = 10000;
        autoTarget = pp;
        for (int i = 0; i < players.count; i++) {
            int tm = players[i];
            if (tm == p) continue;
            const SpatialState &ts = hum(w, tm).spatial;
            float dur = 0.3f + (ts.position - pp).length() * 0.05f;
            dur = lm::lm_powf(clampf_(dur, 0.0f, 1.0f), 0.7f) * 0.7f;
            Vec3 tp = ts.position + ts.movement * dur;
            float dr = lm::lm_powf(nclamp((tp - manualTarget).length(), 0.0f, 70.0f), 0.8f) * 0.8f;
            float ar = fabsf(angle2d_to((tp - pp).normalized(Vec3(0)), inputDir) / (1.0f * kPi)) * 1.0f;
            if (dr + ar < bestRating) {
                bestRating = dr + ar;
                best = tm;
                autoTarget = tp;
            }
        }
    }
    targetPlayer = best;
    Vec3 autoRel = autoTarget - pp, manualRel = manualTarget - pp;
    if (forcedTarget >= 0 || (fullAutoDir && fullAutoPower)) {
        adb = 1.0;
        apb = 1.0;
    } else {
        float maxDist = 50.0f;
        float distFactor =
            (float)(1.0 - (double)lm::lm_powf(clampf_((autoRel - manualRel).length() / maxDist, 0.0f, 1.0f), 1.5f));
        float prox = lm::lm_powf(1.0f - nclamp((pp - autoTarget).length(), 0.0f, 12.0f), 0.5f);
        if (fullAutoDir) {
            adb = 1.0f;
        } else {
            adb *= distFactor;
            adb = lm::lm_powf(adb, 1.0f - prox * 0.9f);
        }
        if (fullAutoPower) {
            apb = 1.0f;
        } else {
            apb *= distFactor;
            apb = clampf_((float)((double)apb * (1.0 + (double)prox)), 0.0f, 1.0f);
        }
    }
    if (passType == kFtLongPass) {
        float td = autoRel.length() * adb + manualRel.length() * (1.0f - adb);
        Vec3 off = Vec3(-team_side(w, teamID) * td * 0.2f, 0, 0);
        autoRel += off;
        manualRel += off;
    }
    Vec3 rtr = (autoRel.normalized(Vec3(0)) * adb + manualRel.normalized(Vec3(0)) * (1.0f - adb))
                   .normalized(manualTarget);
    rtr *= float(autoRel.length() * apb + manualRel.length() * (1.0f - apb));
    auto_pass(passType, rtr, outDir, outPower);
}
CB_HDNI Vec3 shot_direction(const Match &w, int p, const Vec3 &inputDir, float autoDirBias) {
    const SpatialState &sp = hum(w, p).spatial;
    const int side = team_side(w, w.playerTeamID[p]);
    Vec3 manual = inputDir;
    Vec3 goal = Vec3(side * -kPitchHalfL, 0, 0);
    Vec3 toGoal = (goal - (sp.position + sp.movement * 0.12f)).normalized(Vec3(0));
    float rel = angle2d_to(toGoal, inputDir);
    float sideF = clampf_((rel / kPi) / 0.5f, -1.0f, 1.0f);
    sideF = lm::lm_powf(fabsf(sideF), 0.7f) * sign_side(sideF);
    goal.c[1] = sideF * kGoalHalfW * 0.9f * side;
    Vec3 autoDir = (goal - (sp.position + sp.movement * 0.12f)).normalized(Vec3(0));
    return (manual * (1.0f - autoDirBias) + autoDir * autoDirBias).normalized(inputDir);
}

// ---------------------------------------------------------------------------------------------
// Keyboard input of an externally controlled player.
CB_HD HumanGamer &gamer_of(Match &w, int p) {
    int gi = w.m.players[p].base.externalController;
    int first = w.m.teams[0].gamers.count;
    return gi < first ? w.m.teams[0].gamers[gi] : w.m.teams[1].gamers[gi - first];
}
CB_HD float last_switch_bias(Match &w, ControllerState &c) {
    if (!w.m.inPlay || w.m.inSetPiece) c.lastSwitchTime_ms = (uint64_t)(int64_t)-10000;
    if (c.lastSwitchTimeDuration_ms > 0)
        return 1.0f - clampf_((w.m.actualTime_ms - c.lastSwitchTime_ms) / (float)c.lastSwitchTimeDuration_ms,
                              0.0f, 1.0f);
    return 0.0f;
}
CB_HDNI void keyboard_input(Match &w, int p, Vec3 &dir, float &vel) {
    HumanControllerState &hc = gamer_of(w, p).controller;
    const SpatialState &sp = hum(w, p).spatial;
    dir = hc.keyboard.direction;
    const Vec3 pos = sp.position;
    float &dx = dir.c[0], &dy = dir.c[1];
    // Equal to std::min(0.0f, x) / std::max(0.0f, x) with signed zeros; `+ 0.0f` keeps an input -0
    // from surviving a compiler min on the device.
    if (pos.c[0] > kPitchHalfL) dx = ((dx < 0.0f) ? dx : 0.0f) + 0.0f;
    if (pos.c[0] < -kPitchHalfL) dx = (0.0f < dx) ? dx : 0.0f;
    if (pos.c[1] > kPitchHalfW) dy = ((dy < 0.0f) ? dy : 0.0f) + 0.0f;
    if (pos.c[1] < -kPitchHalfW) dy = (0.0f < dy) ? dy : 0.0f;
    if (dir.length() < kStickDeadzone) {
        dir = sp.directionVector;
        vel = kIdleVel;
    } else {
        const bool *b = hc.keyboard.buttons;
        if (b[kBtnSprint]) vel = kSprintVel;
        else if (b[kBtnDribble]) vel = kDribbleVel;
        else if (b[kBtnSwitch] && w.m.designatedPossessionPlayer == p) vel = kIdleVel;
        else vel = kWalkVel;
        dir.normalize();
    }
    if (last_switch_bias(w, hc.base) > 0.0f) {
        float influence = 0.5f;
        float sb = lm::lm_powf(last_switch_bias(w, hc.base), 0.7f);
        Vec3 cur = sp.directionVector * player_float_velocity(w, p);
        Vec3 man = dir * vel;
        Vec3 res = cur * sb * influence + man * (1.0f - sb * influence);
        dir = res.normalized(dir);
        vel = res.length();
    }
}
CB_HD float keyboard_velocity(Match &w, int p) {
    Vec3 d;
    float v = 0;
    keyboard_input(w, p, d, v);
    return v;
}
CB_HD Vec3 keyboard_direction(Match &w, int p) {
    return gamer_of(w, p).controller.keyboard.direction.normalized(hum(w, p).spatial.directionVector);
}

}  // namespace cb
