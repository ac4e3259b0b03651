// cuju-b200: the reset of a match for a set piece, and the placement of both teams for it.
// The placement keeps every double/float conversion of GRF's arithmetic.
//   cuju include/cuju/simulation/reset.h:17-720
#pragma once

#include "team_ai.cuh"

namespace cb {


/// reset.h:19 (LeftTeamOwnsBall).
CB_HD bool left_team_owns_ball(const Match &w) {
    const Scenario &sc = w.scenario;
    float l = 1000000, r = 1000000;
    for (int p = 0; p < sc.leftTeamSize; p++) l = std_min(l, (sc.leftTeam[p].startPosition - sc.ballPosition).length());
    for (int p = 0; p < sc.rightTeamSize; p++)
        r = std_min(r, (sc.rightTeam[p].startPosition - sc.ballPosition).length());
    return l < r;
}

/// reset.h:42 (HumanoidResetPosition). `h` counts players first, then officials.
CB_HDNI bool humanoid_reset_position(const Sim &s, int h, const Vec3 &np, const Vec3 &focus) {
    Match &w = s.w;
    Humanoid &hu = any_hum(w, h);
    SpatialState &sp = hu.spatial;
    hu.startPosition = np;
    set_radian(hu.startAngle, fix_angle(angle2d((focus - np).normalized(Vec3(0, -1, 0)))));
    hu.nextStartPosition = hu.startPosition;
    hu.nextStartAngle = hu.startAngle;
    hu.previousPosition2D = hu.startPosition;
    sp.position = hu.startPosition;
    sp.angle = hu.startAngle;
    sp.directionVector = rot2d(Vec3(0, -1, 0), hu.startAngle.value());
    sp.floatVelocity = 0;
    sp.actualMovement = Vec3(0);
    sp.physicsMovement = Vec3(0);
    sp.animationMovement = Vec3(0);
    sp.movement = Vec3(0);
    sp.actionSmuggleMovement = Vec3(0);
    sp.movementSmuggleMovement = Vec3(0);
    sp.positionOffsetMovement = Vec3(0);
    set_radian(sp.relBodyAngleNonQuantized, 0);
    sp.velocityCategory = kVelIdle;
    sp.relBodyDirectionVector = Vec3(0, -1, 0);
    set_radian(sp.relBodyAngle, 0);
    sp.bodyDirectionVector = Vec3(0, -1, 0);
    set_radian(sp.bodyAngle, 0);
    sp.foot = kFootRight;

    Selector sel(s, h);
    const int idle = sel.idle_movement_animation();
    if (*s.status) return false;
    const Anim &a = s.A(idle);
    AnimationState &ca = hu.anim;
    ca.id = idle;
    ca.anim = idle;
    ca.positions.count = a.positionCount;
    crew_copy_words(reinterpret_cast<uint32_t *>(ca.positions.el),
                   reinterpret_cast<const uint32_t *>(s.T().positions + a.firstPosition), 3 * a.positionCount);
    // The frame draws below the effective frame count, one less than the frame count.
    ca.frameNumber = cvt_f_i32(random_in_range(w.rng, 0, (float)(a.frameCount - 1 - 1)));
    ca.touchFrame = -1;
    ca.originatingInterrupt = kIntNone;
    ca.actionSmuggle = Vec3(0);
    ca.actionSmuggleOffset = Vec3(0);
    ca.actionSmuggleSustain = Vec3(0);
    ca.actionSmuggleSustainOffset = Vec3(0);
    ca.movementSmuggle = Vec3(0);
    ca.movementSmuggleOffset = Vec3(0);
    set_radian(ca.rotationSmuggle.begin, 0);
    set_radian(ca.rotationSmuggle.end, 0);
    set_radian(ca.rotationSmuggleOffset, 0);
    ca.functionType = kFtMovement;
    ca.incomingMovement = Vec3(0);
    ca.outgoingMovement = Vec3(0);
    ca.positionOffset = Vec3(0);
    hu.prevAnimFrameNumber = 0;
    hu.prevAnimFunctionType = kFtMovement;
    hu.nodes[0].position = hu.startPosition;
    hu.applyBuffer.anim = ca.anim;
    hu.applyBuffer.smooth = false;
    hu.applyBuffer.smoothFactor = 0.0f;
    hu.applyBuffer.position = hu.startPosition;
    hu.applyBuffer.orientation = hu.startAngle;
    hu.interruptAnim = kIntNone;
    hu.tripType = 0;
    hu.decayingPositionOffset = Vec3(0);
    hu.decayingDifficultyFactor = 0.0f;
    hu.movementHistory.count = 0;
    hu.requeueDelayFrames = 0;
    hu.tripDirection = Vec3(0);
    const Skeleton &sk = s.ctx.skeletons[h];
    for (int bp = 0; bp < kBodyParts - 1; bp++) hu.nodes[sk.nodeMap[bp]].rotation = Quat();
    return true;
}

/// reset.h:127 (HumanoidSelectRetainAnimation): the throw-in taker's ball-holding animation.
CB_HDNI bool humanoid_select_retain_animation(const Sim &s, int h) {
    Match &w = s.w;
    Humanoid &hu = any_hum(w, h);
    Selector sel(s, h);
    CrudeQuery q;
    q.byFunctionType = true;
    q.functionType = kFtMovement;
    q.byIncomingVelocity = true;
    q.incomingVelocity = kVelIdle;
    q.byOutgoingVelocity = true;
    q.outgoingVelocity = kVelIdle;
    q.incomingRetainState = kSS_RightElbow;
    AnimList l;
    crude_selection(s, q, l);
    if (l.count == 0) return s.fail(kStatusUnsupported);
    sel.set_movement_predicate(Vec3(0, -1, 0), kVelIdle);
    sel.sort(l, [&](int i) { return sel.movement_similarity_key(i); });
    set_radian(hu.startAngle, fix_angle(angle2d(Vec3(0) - hu.startPosition)));
    AnimationState &ca = hu.anim;
    ca.positions.count = 0;
    ca.anim = l[0];
    ca.id = l[0];
    ca.frameNumber = 0;
    ca.touchFrame = -1;
    ca.actionSmuggle = Vec3(0);
    ca.actionSmuggleOffset = Vec3(0);
    ca.actionSmuggleSustain = Vec3(0);
    ca.actionSmuggleSustainOffset = Vec3(0);
    ca.movementSmuggle = Vec3(0);
    ca.movementSmuggleOffset = Vec3(0);
    set_radian(ca.rotationSmuggle.begin, 0);
    set_radian(ca.rotationSmuggle.end, 0);
    set_radian(ca.rotationSmuggleOffset, 0);
    ca.functionType = kFtMovement;
    hu.applyBuffer.anim = ca.anim;
    hu.applyBuffer.smooth = false;
    hu.applyBuffer.position = hu.startPosition;
    hu.applyBuffer.orientation = hu.startAngle;
    w.m.ballRetainer = h;
    return true;
}

/// reset.h:175 (PlayerBaseResetSituation).
template <class C>
CB_HDNI bool person_reset_situation(const Sim &s, PersonBase<C> &b, int h, const Vec3 &focus) {
    b.positionHistoryPerSecond.count = 0;
    b.lastTouchTime_ms = 0;
    b.lastTouchType = kTouchNone;
    if (b.isActive) {
        b.humanoid.mentalImageTime = 0;
        Vec3 p = b.humanoid.spatial.position;
        if (!humanoid_reset_position(s, h, p, focus)) return false;
    }
    return true;
}
CB_HDNI bool player_base_reset_situation(const Sim &s, int h, const Vec3 &focus) {
    Match &w = s.w;
    const int pc = w.m.playerCount;
    if (h < pc) {
        PersonBase<AIControllerState> &b = w.m.players[h].base;
        if (!person_reset_situation(s, b, h, focus)) return false;
        if (external_active(w, h)) {
            human_controller_reset(w, b.externalController);
        } else {
            b.controller.lastDesiredDirection = Vec3(0);
            b.controller.lastDesiredVelocity = 0;
        }
        return true;
    }
    return person_reset_situation(s, w.m.officials[h - pc], h, focus);
}

/// reset.h:220 (PlayerResetSituation).
CB_HDNI bool player_reset_situation(const Sim &s, int p, const Vec3 &focus) {
    if (!player_base_reset_situation(s, p, focus)) return false;
    Player &pl = s.w.m.players[p];
    pl.hasPossession = false;
    pl.hasBestPossession = false;
    pl.hasUniquePossession = false;
    pl.possessionDuration_ms = 0;
    pl.timeNeededToGetToBall_ms = 1000;
    pl.timeNeededToGetToBallOptimistic_ms = 1000;
    pl.desiredTimeToBall_ms = 0;
    pl.manMarking = -1;
    pl.triggerControlledBallCollision = false;
    pl.tactical.forwardSpaceRating = 0;
    pl.tactical.toGoalSpaceRating = 0;
    pl.tactical.spaceRating = 0;
    return true;
}

/// reset.h:238 (TeamAIReset).
CB_HD void team_ai_reset(TeamAIState &t) {
    t.taker = -1;
    t.setPieceType = kGmNormal;
    t.offsideTrapX = 0;
    t.endApplyAttackingRun_ms = 0;
    t.attackingRunPlayer = -1;
    t.endApplyTeamPressure_ms = 0;
    t.teamPressurePlayer = -1;
    t.endApplyKeeperRush_ms = 0;
    t.teamHasPossession = false;
    t.teamHasUniquePossession = false;
    t.oppTeamHasPossession = false;
    t.oppTeamHasUniquePossession = false;
    t.teamHasBestPossession = false;
    t.teamPossessionAmount = 1.0f;
    t.fadingTeamPossessionAmount = 1.0f;
    t.timeNeededToGetToBall = 100;
    t.oppTimeNeededToGetToBall = 100;
}

/// reset.h:266 (TeamResetSituation).
CB_HDNI bool team_reset_situation(const Sim &s, int teamID, const Vec3 &focus) {
    Match &w = s.w;
    Team &t = team_by_id(w, teamID);
    t.timeNeededToGetToBall_ms = 100;
    t.hasPossession = false;
    t.teamPossessionAmount = 1.0f;
    t.fadingTeamPossessionAmount = 1.0f;
    t.lastTouchPlayer = -1;
    PlayerList ps;
    all_players(ps, w, teamID);
    if (ps.count == 0) return s.fail(kStatusUnsupported);
    t.designatedTeamPossessionPlayer = ps[0];
    for (int i = 0; i < ps.count; i++)
        if (w.m.players[ps[i]].base.isActive && !player_reset_situation(s, ps[i], focus)) return false;
    team_ai_reset(t.ai);
    return true;
}

/// reset.h:284 (BallResetSituation).
CB_HDNI void ball_reset_situation(Ball &b, const Vec3 &focus) {
    ball_materialize(b);
    b.momentum = Vec3(0);
    b.rotationPerMs = Quat();
    const Vec3 p = focus + Vec3(0, 0, 0.11f);
    crew_for(kPredictionSpan_ms / 10, [&](int i) { b.predictions[i] = p; });
    b.orientationPrediction = Quat();
    b.positionHistory.count = 0;
    b.positionBuffer = p;
    b.validPredictions = 0;
    b.orientationBuffer = Quat();
    b.touchesNet = false;
}

/// reset.h:301 (MatchResetSituation).
CB_HDNI bool match_reset_situation(const Sim &s, const Vec3 &focus) {
    Match &w = s.w;
    MatchState &m = w.m;
    m.cameraPosition.count = 0;
    m.ballRetainer = -1;
    m.ballIsInGoal = false;
    m.goalScored = false;
    m.mentalImages.count = 0;
    for (int i = 0; i < 4; i++) m.lastTouchTeamIDs[i] = -1;
    m.lastTouchTeamID = -1;
    m.lastGoalScorer = -1;
    m.bestPossessionTeam = -1;
    m.possessionSideHistory.count = 0;
    m.lastBodyBallCollisionTime_ms = 0;
    ball_reset_situation(m.ball, focus);
    const int first = w.firstTeamID();
    if (!team_reset_situation(s, first, focus)) return false;
    if (!team_reset_situation(s, 1 - first, focus)) return false;
    return player_base_reset_situation(s, m.playerCount + 0, focus);
}

/// reset.h:326 (TeamAIPrepareSetPiece).
CB_HDNI bool team_ai_prepare_set_piece(const Sim &s, int teamID, int setPiece, int otherTeamID, int kickoffTakerTeamID,
                                       int takerTeamID) {
    Match &w = s.w;
    MatchState &m = w.m;
    Team &team = team_by_id(w, teamID);
    TeamAIState &ai = team.ai;
    const int side = team_side(w, teamID);
    auto flat_ball = [&]() { return ball_predict(m.ball, 0).flat(); };
    auto reset_pos = [&](int p, const Vec3 &pos, const Vec3 &focus) { return humanoid_reset_position(s, p, pos, focus); };
    ai.setPieceType = setPiece;
    if (setPiece == kGmNormal) return true;
    PlayerList players;
    active_players(players, w, teamID);
    for (int i = 0; i < players.count;) {
        Vec3 focus = flat_ball();
        if (formation(s, players[i]).role == kRoleGK) {
            if (setPiece == kGmKickOff) {
                focus.c[0] = 0;
                focus.c[1] = 0;
            }
            if (!reset_pos(players[i], Vec3((float)((double)(kPitchHalfL * side) * 0.98), 0, 0), focus)) return false;
            players.erase_at(i);
        } else {
            i++;
        }
    }
    const bool taker = takerTeamID == teamID;
    team.fadingTeamPossessionAmount = taker ? 1.5f : 0.5f;
    const double dside = side, halfL = kPitchHalfL, halfW = kPitchHalfW;
    auto F = [](double v) { return (float)v; };
    switch (setPiece) {
        case kGmKickOff:
            for (int i = 0; i < players.count; i++) {
                const Vec3 &fp = formation(s, players[i]).position;
                Vec3 bp = fp * Vec3(F((double)(-side * kPitchHalfL) * 0.6), F((double)(-side * kPitchHalfW) * 0.6), 0);
                bp.c[1] += random_in_range(w.rng, -2.0f, 2.0f);
                bp.c[0] = F(bp.c[0] * 0.5);
                bp.c[0] = F(bp.c[0] + (halfL * 0.2) * dside);
                if ((double)(bp.c[0] * side) < 0.5) bp.c[0] = F(0.5 * dside);
                if ((double)bp.length() < 9.4) {
                    bp.normalize(Vec3(side, 0, 0));
                    bp *= 9.4f;
                }
                if (!reset_pos(players[i], bp, flat_ball())) return false;
                if (taker) {
                    PlayerList r;
                    closest_players(r, s, teamID, Vec3(0), false, 2);
                    for (int k = 0; k < r.count; k++)
                        if (!reset_pos(r[k], Vec3(0, F((double)k * 1.4 * dside), 0), flat_ball())) return false;
                }
            }
            break;
        case kGmGoalKick:
            for (int i = 0; i < players.count; i++) {
                float back, front;
                if (taker) {
                    back = F((double)(side * kPitchHalfL) * 0.5);
                    front = F((double)(-side * kPitchHalfL) * 0.2);
                } else {
                    back = F((double)(side * kPitchHalfL) * 0.4);
                    front = F((double)(-side * kPitchHalfL) * 0.1);
                }
                float lowY = F(-halfW * 0.7), highY = F(halfW * 0.7);
                Vec3 bp = adapted_formation_position(s, players[i], back, front, lowY, highY, 0, 0, 0, 0, Vec3(0), 0,
                                                     0, 0, false);
                if (!reset_pos(players[i], bp, flat_ball())) return false;
            }
            break;
        case kGmCorner:
            for (int i = 0; i < players.count; i++) {
                float back, front, xF, xFS, yF, yFS, midF, midFS;
                Vec3 b = flat_ball();
                if (taker) {
                    back = F((double)(-side * kPitchHalfL) * 0.2);
                    front = F((double)(-side * kPitchHalfL) * 0.96);
                    xF = F(front * 0.85);
                    xFS = 0.7f;
                    yF = b.c[1] * 0.1f;
                    yFS = 0.7f;
                    midF = 0.9f;
                    midFS = 0.5f;
                } else {
                    back = F((double)(side * kPitchHalfL) * 0.98);
                    front = F((double)(side * kPitchHalfL) * 0.5);
                    xF = F(back * 0.94);
                    xFS = 0.8f;
                    yF = b.c[1] * 0.1f;
                    yFS = 0.9f;
                    midF = 0.1f;
                    midFS = 0.7f;
                }
                float lowY = F(-halfW * 0.6), highY = F(halfW * 0.6);
                Vec3 bp = adapted_formation_position(s, players[i], back, front, lowY, highY, xF, xFS, yF, yFS,
                                                     Vec3(b.c[0] * 0.95f, b.c[1] * 0.1f, 0), 0.9f, midF, midFS, false);
                if (!reset_pos(players[i], bp, flat_ball())) return false;
            }
            break;
        case kGmThrowIn:
            for (int i = 0; i < players.count; i++) {
                float back, front, xF, xFS, yF, yFS;
                Vec3 b = flat_ball();
                if (taker) {
                    back = clampf_(b.c[0] + 30 * side, -kPitchHalfL, kPitchHalfL);
                    front = clampf_(b.c[0] + 20 * -side, -kPitchHalfL, kPitchHalfL);
                    xF = clampf_(b.c[0] + 4 * -side, -kPitchHalfL, kPitchHalfL);
                    xFS = F(0.4);
                    yF = F(b.c[1] * 0.996);
                    yFS = F(0.6);
                } else {
                    back = clampf_(b.c[0] + 30 * side, -kPitchHalfL, kPitchHalfL);
                    front = clampf_(b.c[0] + 15 * -side, -kPitchHalfL, kPitchHalfL);
                    xF = clampf_(b.c[0] + 16 * side, -kPitchHalfL, kPitchHalfL);
                    xFS = F(0.2);
                    yF = F(b.c[1] * 0.95);
                    yFS = F(0.5);
                }
                float lowY = -kPitchHalfW * 0.75f + b.c[1] * 0.25f;
                float highY = kPitchHalfW * 0.75f + b.c[1] * 0.25f;
                Vec3 bp = adapted_formation_position(s, players[i], back, front, lowY, highY, xF, xFS, yF, yFS, b,
                                                     F(0.7), 0, 0, false);
                if (!reset_pos(players[i], bp, flat_ball())) return false;
            }
            break;
        case kGmFreeKick: {
            for (int i = 0; i < players.count; i++) {
                float back, front, xF, xFS, yF, yFS;
                Vec3 b = flat_ball();
                const float shw = side * kPitchHalfL;
                float xo = F((double)clampf_((b.c[0] * -side) / kPitchHalfL, F(-1.0), F(1.0)) * 0.5 + 0.5);
                if (taker) {
                    back = clampf_(F((double)shw * (0.7 - (double)xo * 0.7)), -kPitchHalfL, kPitchHalfL);
                    front = clampf_(F((double)shw * (-0.3 - (double)xo * 0.7)), -kPitchHalfL, kPitchHalfL);
                    xF = clampf_(b.c[0] + 10 * -side, -kPitchHalfL, kPitchHalfL);
                    xFS = F(0.5 + (double)xo * 0.2);
                    yF = F(b.c[1] * 0.4);
                    yFS = F(0.6 + (double)xo * 0.2);
                } else {
                    back = clampf_(F((double)shw * (1.0 - (double)xo * 0.6)), -kPitchHalfL, kPitchHalfL);
                    front = clampf_(F((double)shw * (0.5 - (double)xo * 0.8)), -kPitchHalfL, kPitchHalfL);
                    xF = clampf_(b.c[0] + 20 * side, -kPitchHalfL, kPitchHalfL);
                    xFS = F(0.6 - (double)xo * 0.4);
                    yF = F(b.c[1] * 0.2);
                    yFS = F(0.8 - (double)xo * 0.4);
                }
                float lowY = F(-halfW * 0.7), highY = F(halfW * 0.7);
                Vec3 bp = adapted_formation_position(s, players[i], back, front, lowY, highY, xF, xFS, yF, yFS, b,
                                                     F(0.4), 0, 0, false);
                if (!taker) {
                    if ((double)(bp - flat_ball()).length() < 9.15)
                        bp = flat_ball() + (bp - flat_ball()).normalized() * 9.15f;
                }
                if (!reset_pos(players[i], bp, flat_ball())) return false;
            }
            if (!taker && (double)(flat_ball() - Vec3(side * kPitchHalfL, 0, 0)).length() < 40.0) {
                PlayerList r;
                closest_players(r, s, teamID, flat_ball(), false, 3);
                for (int k = 0; k < r.count; k++) {
                    Vec3 tg = (Vec3(side * kPitchHalfL, 0, 0) - flat_ball()).normalized(Vec3(0));
                    tg += Vec3(0, F(1.0 - (double)k), 0) * F(0.07);
                    tg.normalize();
                    if (!reset_pos(r[k], flat_ball() + tg * 9.15f, flat_ball())) return false;
                }
            }
            break;
        }
        case kGmPenalty:
            for (int i = 0; i < players.count; i++) {
                float back, front, xF, xFS, yF, yFS;
                Vec3 b = flat_ball();
                if (taker) {
                    back = clampf_(b.c[0] + 50 * side, -kPitchHalfL, kPitchHalfL);
                    front = clampf_(b.c[0] + 10 * -side, -kPitchHalfL, kPitchHalfL);
                    xF = b.c[0];
                    xFS = F(0.6);
                    yF = F(0.0);
                    yFS = F(0.8);
                } else {
                    back = clampf_(b.c[0] + 11 * side, -kPitchHalfL, kPitchHalfL);
                    front = clampf_(b.c[0] + 20 * -side, -kPitchHalfL, kPitchHalfL);
                    xF = b.c[0];
                    xFS = F(1.0);
                    yF = F(0.0);
                    yFS = F(1.0);
                }
                float lowY = F(-halfW * 0.8), highY = F(halfW * 0.8);
                Vec3 bp = adapted_formation_position(s, players[i], back, front, lowY, highY, xF, xFS, yF, yFS, Vec3(0),
                                                     0, 0, 0, false);
                int ps = (ball_predict(m.ball, 0).c[0] < 0) ? -1 : 1;
                if ((double)(bp.c[0] * ps) > halfL - 16.5 - 0.5) bp.c[0] = F((halfL - 16.5 - 0.5) * ps);
                if ((double)(bp - flat_ball()).length() < 9.15 + 0.5)
                    bp = flat_ball() + (bp - flat_ball()).normalized() * F(9.15 + 0.5);
                if (!reset_pos(players[i], bp, flat_ball())) return false;
            }
            break;
        default:
            for (int i = 0; i < players.count; i++) {
                Vec3 bp = formation(s, players[i]).position *
                          Vec3(F((double)(-side * kPitchHalfL) * 0.7), F((double)(-side * kPitchHalfW) * 0.7), 0);
                if (!reset_pos(players[i], bp, flat_ball())) return false;
            }
            break;
    }

    if (setPiece == kGmKickOff) {
        PlayerList fps;
        all_players(fps, w, teamID);
        PlayerList tps;
        all_players(tps, w, teamID);
        // After the start, a kickoff to the team that did not own the ball at the start swaps the
        // start positions of equal-sized teams.
        if (m.matchTime_ms > 0 && team_count(w, otherTeamID) == fps.count &&
            (left_team_owns_ball(w) ^ (kickoffTakerTeamID == 0)))
            all_players(fps, w, otherTeamID);
        for (int i = 0; i < fps.count; i++) {
            if (!m.players[tps[i]].base.isActive) continue;
            Vec3 bp = formation(s, fps[i]).startPosition * Vec3(-side * kPitchHalfL, -side * kPitchHalfW, 0);
            if (!reset_pos(tps[i], bp, flat_ball())) return false;
        }
    }

    if (taker) {
        Vec3 b = flat_ball();
        PlayerList cl;
        closest_players(cl, s, teamID, flat_ball(), false, 2);
        if (cl.count == 0) return s.fail(kStatusUnsupported);
        ai.taker = cl[0];
        if (setPiece == kGmKickOff) {
            // The kickoff taker keeps its formation position.
        } else if (setPiece == kGmThrowIn) {
            if (!reset_pos(cl[0], b + flat_ball().normalized(Vec3(0, -side, 0)) * 0.3f, b)) return false;
        } else if (setPiece == kGmFreeKick) {
            if (!reset_pos(ai.taker, b + Vec3(side, 0, 0) * 2.3f, b)) return false;
        } else {
            if (!reset_pos(ai.taker, b + flat_ball().normalized(Vec3(0, -side, 0)) * 2.3f, b)) return false;
        }
        if (setPiece == kGmThrowIn && !humanoid_select_retain_animation(s, ai.taker)) return false;
        if (setPiece == kGmPenalty) {
            if (!reset_pos(ai.taker, b + Vec3(side, 0, 0) * 3.0f, b)) return false;
        }
    } else {
        ai.taker = -1;
    }
    return true;
}

/// reset.h:625 (PlayerSendOff).
CB_HDNI bool player_send_off(const Sim &s, int p) {
    Match &w = s.w;
    MatchState &m = w.m;
    Player &pl = m.players[p];
    const int teamID = w.playerTeamID[p];
    random_in_range(w.rng, 0, 3);  // the referee's message draws once
    auto cur = [&]() { return pl.base.humanoid.spatial.position; };
    if (!player_reset_situation(s, p, cur())) return false;
    if (pl.base.externalController >= 0) {
        Team &t = team_by_id(w, teamID);
        for (int g = 0; g < t.gamers.count; g++) {
            if (t.gamers.el[g].selectedPlayer != p) continue;
            int some = closest_player(s, teamID, cur(), true, p, true);
            t.mainSelectedPlayer = some;
            gamer_set_selected(w, global_gamer(w, teamID, g), some);
        }
    }
    // The deactivation resets the player a second time.
    if (!player_reset_situation(s, p, cur())) return false;
    pl.base.isActive = false;
    pl.base.externalController = -1;
    team_by_id(w, teamID).designatedTeamPossessionPlayer =
        closest_player(s, teamID, ball_predict(m.ball, 0).flat(), false);
    if (formation(s, p).role == kRoleGK) {
        int first = -1;
        for (int c = 0; c < m.playerCount && first < 0; c++)
            if (w.playerTeamID[c] == teamID && m.players[c].base.isActive) first = c;
        if (first < 0) return s.fail(kStatusUnsupported);
        w.formationOverride[first] = (int8_t)(1 + formation_source(w, p));
    }
    return true;
}

/// reset.h:664 (RefereePrepareSetPiece).
CB_HDNI bool referee_prepare_set_piece(const Sim &s, int setPiece) {
    Match &w = s.w;
    Referee &ref = w.m.referee;
    RefereeBuffer &buf = ref.buffer;
    if (setPiece == kGmFreeKick) {
        buf.restartPosition.c[0] =
            clampf_(buf.restartPosition.c[0], (float)(-0.95 * kPitchHalfL), (float)(0.95 * kPitchHalfL));
        buf.restartPosition.c[1] =
            clampf_(buf.restartPosition.c[1], (float)(-0.95 * kPitchHalfW), (float)(0.95 * kPitchHalfW));
    }
    if (!match_reset_situation(s, w.scenario.reverseTeamProcessing ? -buf.restartPosition : buf.restartPosition))
        return false;
    const int first = w.firstTeamID(), second = 1 - first;
    const int spTeam = buf.setPieceTeam == 0 ? first : second;
    if (!team_ai_prepare_set_piece(s, first, setPiece, second, spTeam, buf.teamID)) return false;
    if (!team_ai_prepare_set_piece(s, second, setPiece, first, spTeam, buf.teamID)) return false;
    buf.taker = team_by_id(w, buf.teamID).ai.taker;
    ref.offsidePlayers.count = 0;
    return true;
}

}  // namespace cb
