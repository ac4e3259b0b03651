// cuju-b200: gamer/player selection of a team and the per-tick process of a player's humanoid
// (next frame, interrupts, command -> animation, ball touches, smuggle offsets).
//   gamer selection    cuju include/cuju/simulation/team_select.h:17-204
//   humanoid tick      cuju include/cuju/simulation/humanoid_process.h:23-678
#pragma once

#include "skeleton.cuh"
#include "touch.cuh"

namespace cb {

using CommandQueue = List<PlayerCommand, 16>;

// Global gamer index: gamers of the team processed first come first.
CB_HD int global_gamer(const Match &w, int teamID, int g) {
    return team_slot(w, teamID) == 0 ? g : w.m.teams[0].gamers.count + g;
}
CB_HD HumanGamer &gamer_global(Match &w, int gi) {
    int first = w.m.teams[0].gamers.count;
    return gi < first ? w.m.teams[0].gamers[gi] : w.m.teams[1].gamers[gi - first];
}
// Releases the non-sticky buttons of both stored copies of a gamer's keyboard.
CB_HD void release_nonsticky(Match &w, int gi) {
    Keyboard *kbs[2] = {&gamer_global(w, gi).controller.keyboard, &w.m.secondKeyboardCopies[gi]};
    const int btns[6] = {kBtnLongPass, kBtnHighPass, kBtnShortPass, kBtnShot, kBtnSliding, kBtnSwitch};
    for (int k = 0; k < 2; k++)
        for (int b = 0; b < 6; b++) kbs[k]->buttons[btns[b]] = false;
}
CB_HDNI void human_controller_reset(Match &w, int gi) {
    HumanControllerState &c = gamer_global(w, gi).controller;
    c.actionMode = 0;
    c.gauge_ms = 0;
    c.actionButton = kBtnShortPass;
    c.actionBufferTime_ms = 0;
    c.base.lastSwitchTime_ms = (uint64_t)(int64_t)-10000;
    c.base.lastSwitchTimeDuration_ms = 300;
    c.lastSteadyDirectionSnapshotTime_ms = 0;
    c.steadyDirection = Vec3(0, -1, 0);
    c.previousDirection = Vec3(0, -1, 0);
    c.base.fadingTeamPossessionAmount = 1.0;
    release_nonsticky(w, gi);
}
CB_HD void human_controller_set_player(Match &w, int gi, int p) {
    HumanControllerState &c = gamer_global(w, gi).controller;
    c.base.lastSwitchTime_ms = w.m.actualTime_ms;
    c.base.player = p;
    c.base.team = team_slot(w, w.playerTeamID[p]);
    c.base.opponentTeam = team_slot(w, 1 - w.playerTeamID[p]);
}
CB_HD void set_external_controller(Match &w, int p, int gi) {
    Player &pl = w.m.players[p];
    pl.base.externalController = gi;
    if (gi >= 0) {
        human_controller_reset(w, gi);
        human_controller_set_player(w, gi, p);
    } else {
        pl.base.controller.lastDesiredDirection = Vec3(0);
        pl.base.controller.lastDesiredVelocity = 0;
    }
}
CB_HDNI void gamer_set_selected(Match &w, int gi, int p) {
    HumanGamer &g = gamer_global(w, gi);
    if (p >= 0 && w.m.players[p].base.externalController >= 0) return;
    if (g.selectedPlayer >= 0) {
        if (g.selectedPlayer == p) return;
        set_external_controller(w, g.selectedPlayer, -1);
    }
    if (p >= 0) {
        g.selectedPlayer = p;
        set_external_controller(w, p, gi);
    } else {
        g.selectedPlayer = -1;
    }
}
CB_HDNI bool team_select_player(const Sim &s, int teamID, int p) {
    Match &w = s.w;
    Team &t = team_by_id(w, teamID);
    if (formation(s, p).controllable) {
        t.mainSelectedPlayer = p;
        if (w.m.players[p].base.externalController < 0 && t.gamers.count > 0) {
            auto &sp = t.switchPriority;
            int g = sp[0];
            gamer_set_selected(w, global_gamer(w, teamID, g), p);
            for (int i = 0; i + 1 < sp.count; i++) sp[i] = sp[i + 1];
            sp[sp.count - 1] = g;
        }
    }
    t.designatedTeamPossessionPlayer = p;
    return true;
}
// A tie keeps the player that comes first in the state.
CB_HDNI int closest_player(const Sim &s, int teamID, const Vec3 &pos, bool onlyAI, int except = -1,
                           bool onlySelectable = false) {
    const Match &w = s.w;
    float cd = 10000;
    int cp = -1;
    for (int p = 0; p < w.m.playerCount; p++) {
        if (w.playerTeamID[p] != teamID) continue;
        if (!w.m.players[p].base.isActive || p == except) continue;
        float d = (hum(w, p).spatial.position - pos).length();
        if (d < cd) {
            if ((!onlyAI || !external_active(w, p)) && (!onlySelectable || formation(s, p).controllable)) {
                cd = d;
                cp = p;
            }
        }
    }
    return cp;
}
// The shortest time to the ball (ms) of the players the enabled gamers control, or 10000.
CB_HD int human_time_to_ball(const Match &w, int teamID) {
    const Team &t = team_by_id(w, teamID);
    int tt = 10000;
    for (int g = 0; g < t.gamers.count; g++) {
        const HumanGamer &hg = t.gamers[g];
        if (hg.selectedPlayer >= 0 && !hg.controller.keyboard.disabled) {
            int v = (int)w.m.players[hg.selectedPlayer].timeNeededToGetToBall_ms;
            tt = (v < tt) ? v : tt;
        }
    }
    return tt;
}
CB_HDNI bool team_update_switch(const Sim &s, int teamID) {
    Match &w = s.w;
    MatchState &m = w.m;
    Team &t = team_by_id(w, teamID);
    if (m.inPlay && t.gamers.count > 1) {
        auto &sp = t.switchPriority;
        int mine = sp[0];
        if (t.gamers[mine].selectedPlayer == m.designatedPossessionPlayer) {
            for (int i = 0; i + 1 < sp.count; i++) sp[i] = sp[i + 1];
            sp[sp.count - 1] = mine;
        }
    }
    if (m.inPlay && t.gamers.count > 0) {
        int d = t.designatedTeamPossessionPlayer;
        if (!external_active(w, d) &&
            3 * (int)m.players[d].timeNeededToGetToBall_ms < human_time_to_ball(w, teamID) &&
            formation(s, d).role != kRoleGK) {
            if (!team_select_player(s, teamID, d)) return false;
        }
    }
    if (m.inPlay && t.gamers.count > 0) {
        int d = t.designatedTeamPossessionPlayer;
        if (!external_active(w, d) && (m.players[d].hasUniquePossession || m.inSetPiece)) {
            if (formation(s, d).role != kRoleGK) {
                if (!team_select_player(s, teamID, d)) return false;
            }
        }
    }
    return true;
}
CB_HDNI void team_gamers_select_anyone(const Sim &s, int teamID) {
    Match &w = s.w;
    if (!w.m.inPlay) return;
    Team &t = team_by_id(w, teamID);
    if (t.mainSelectedPlayer == -1)
        t.mainSelectedPlayer = closest_player(s, teamID, ball_at(w, 0).flat(), true, -1, true);
    for (int g = 0; g < t.gamers.count; g++) {
        if (t.gamers[g].selectedPlayer == -1) {
            int p = closest_player(s, teamID, ball_at(w, 0).flat(), true, -1, true);
            if (p >= 0) gamer_set_selected(w, global_gamer(w, teamID, g), p);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Commands.
// Commands are built through a reference, not returned by value: aggregates returned by value from
// inlined calls were seen to lose their stack slot in the sm_100a build.
CB_HD void default_command(PlayerCommand &c) {
    memset(&c, 0, sizeof(c));
    c.desiredFunctionType = kFtMovement;
    c.useDesiredMovement = false;
    c.desiredVelocityFloat = kIdleVel;
    c.strictMovement = kStrictDynamic;
    c.useDesiredLookAt = false;
    c.useTouchInfo = false;
    c.useTripType = false;
    c.useDesiredTripDirection = false;
    c.onlyDeflectAnimationsThatPickupBall = false;
    c.tripType = 1;
    c.useSpecialVar1 = false;
    c.specialVar1 = 0;
    c.useSpecialVar2 = false;
    c.specialVar2 = 0;
    c.modifier = 0;
    c.touchInfo.targetPlayer = -1;
    c.touchInfo.forcedTargetPlayer = -1;
}
CB_HD void trip_command(PlayerCommand &c, const Humanoid &h, const Vec3 &trip, int tripType) {
    default_command(c);
    c.desiredFunctionType = kFtTrip;
    c.useDesiredMovement = false;
    c.useDesiredTripDirection = true;
    c.desiredTripDirection = trip;
    c.desiredVelocityFloat = h.spatial.floatVelocity;
    c.useTripType = true;
    c.tripType = tripType;
}
CB_HD bool queue_push(const Sim &s, CommandQueue &q, const PlayerCommand &c) {
    if (q.count >= 16) return s.fail(kStatusOverflow);
    q.push(c);
    return true;
}
CB_HD void add_trip_commands(const Sim &s, const Humanoid &h, CommandQueue &q, int tripType) {
    PlayerCommand c;
    if (tripType == 1) {
        trip_command(c, h, h.tripDirection, tripType);
        queue_push(s, q, c);
    } else {
        int other = 3;
        if (tripType == 3) other = 2;
        trip_command(c, h, h.tripDirection, tripType);
        queue_push(s, q, c);
        trip_command(c, h, h.tripDirection, other);
        queue_push(s, q, c);
        trip_command(c, h, h.tripDirection, 1);
        queue_push(s, q, c);
    }
}
CB_HD void basic_movement_command(PlayerCommand &c, const Humanoid &h, float vel) {
    default_command(c);
    c.desiredFunctionType = kFtMovement;
    c.useDesiredMovement = true;
    c.useDesiredLookAt = true;
    c.desiredDirection = h.spatial.directionVector;
    c.desiredVelocityFloat = vel;
    c.desiredLookAt = h.spatial.position + c.desiredDirection * 10.0f;
}

CB_HDNI bool player_request_command(const Sim &s, int p, CommandQueue &q);  // ai_ctrl.cuh

CB_HD Vec3 current_outgoing_movement(const AnimationState &ca) {
    if (ca.positions.count < 2) return Vec3(0);
    return (ca.positions[ca.positions.count - 1] - ca.positions[ca.positions.count - 2]) * 100.0f;
}

// The interrupt branch of a humanoid tick (humanoid_process.h): the command request, the
// animation selection over the queued commands and the new animation's start. Reads and writes
// only the match, so a whole warp can run it for one environment.
CB_HDNI bool humanoid_interrupt(const Sim &s, int p) {
    Humanoid &h = s.w.m.players[p].base.humanoid;
    AnimationState &ca = h.anim;
    CommandQueue q;
    if (h.interruptAnim == kIntTrip && h.tripType != 0) {
        add_trip_commands(s, h, q, h.tripType);
        h.tripType = 0;
        PlayerCommand bmc;
        basic_movement_command(bmc, h, h.spatial.floatVelocity);
        queue_push(s, q, bmc);
    } else {
        q.count = 0;
        if (!player_request_command(s, p, q)) return false;
    }
    bool found = false, preferPass = false;
    for (int i = 0; i < q.count; i++) {
        const PlayerCommand &c = q[i];
        if (c.desiredFunctionType == kFtShortPass || c.desiredFunctionType == kFtLongPass ||
            c.desiredFunctionType == kFtHighPass || c.desiredFunctionType == kFtShot)
            preferPass = true;
        Selector sel(s, p);
        int r = sel.select(c, h.interruptAnim, preferPass);
        if (r == kSelUnsupported) return s.fail(kStatusUnsupported);
        if (*s.status != kStatusOk) return false;
        found = r == kSelTrue;
        if (found) break;
    }
    if (h.interruptAnim == kIntSwitch && !found) return s.fail(kStatusUnsupported);
    if (found) {
        h.startPosition = h.spatial.position;
        h.startAngle = h.spatial.angle;
        {
            Selector sel(s, p);
            Vec3 nsp;
            float nsa;
            sel.predicted_situation(nsp, nsa);
            h.nextStartPosition = nsp;
            set_radian(h.nextStartAngle, nsa);
        }
        h.applyBuffer.anim = ca.anim;
        h.applyBuffer.smooth = true;
        h.applyBuffer.smoothFactor = (h.interruptAnim == kIntSwitch && h.prevAnimFunctionType == kFtMovement &&
                                      ca.functionType == kFtMovement)
                                         ? 0.0f
                                         : 1.0f;
        if (ca.functionType == kFtShot) h.applyBuffer.smoothFactor = 0.8f;
        if (ca.functionType == kFtShortPass || ca.functionType == kFtHighPass) h.applyBuffer.smoothFactor = 0.8f;
        if (ca.functionType == kFtDeflect || ca.functionType == kFtSliding) h.applyBuffer.smoothFactor = 0.8f;
        if (ca.functionType == kFtBallControl || ca.functionType == kFtTrap) h.applyBuffer.smoothFactor = 0.8f;
        float ad = s.D(ca.anim).animDifficultyFactor;
        if (ad > h.decayingDifficultyFactor) h.decayingDifficultyFactor = ad;
        if (h.interruptAnim == kIntReQueue && h.prevAnimFunctionType == ca.functionType) h.requeueDelayFrames = 22;
    }
    return true;
}

// The touch part of a humanoid tick (humanoid_process.h): a controlled collision, the touch at the
// animation's touch frame (trap, control, pass, shot, deflection ...) and the retained ball. Reads
// and writes only the match, so a whole warp can run it for one environment; `arg` is the player
// plus 0x10000 when a controlled collision was triggered this tick.
CB_HDNI bool humanoid_touches(const Sim &s, int arg) {
    const int p = arg & 0xffff;
    const bool ctrlColl = (arg & 0x10000) != 0;
    Match &w = s.w;
    Player &pl = w.m.players[p];
    Humanoid &h = pl.base.humanoid;
    AnimationState &ca = h.anim;
    const int teamID = w.playerTeamID[p];
    const Anim &a = s.A(ca.anim);
    const AnimDerived &d = s.D(ca.anim);
    auto nextBodyAngle = [&]() {
        return h.startAngle.value() + a.outgoingAngle.value() + a.outgoingBodyAngle.value() + ca.rotationSmuggle.end.value();
    };
    if (ctrlColl && ca.touchFrame == -1) {
        Vec3 curMom = w.m.ball.momentum;
        float nba = nextBodyAngle();
        float xr = 0, yr = 0;
        Vec3 tv;
        if (!trap_vector(s, p, h.nextStartPosition, h.nextStartAngle.value(), nba, current_outgoing_movement(ca), ca,
                         ca.frameNumber, h.spatial, h.decayingPositionOffset, xr, yr, tv))
            return false;
        if (ca.originatingCommand.modifier & 1) tv *= 1.35f;
        float bumpy = 0.0f;
        tv = tv * (1.0f - bumpy) + curMom * bumpy;
        ball_touch(s, tv);
        ball_set_rotation(w, xr, yr, 0, 0.2f * (1.0f - bumpy));
        if (!team_set_last_touch(s, p, d.touchType)) return false;
    }
    if (ca.touchFrame == ca.frameNumber) {
        Vec3 desBall;
        for (int k = 0; k < a.footballCount; k++) {
            const FootballKey &fk = s.T().football[a.firstFootball + k];
            if (fk.frame == ca.touchFrame) desBall = fk.position;
        }
        float desH = desBall.c[2];
        float touchable = 0.4f;
        float full = (ball_predict(w.m.ball, 0) - (ca.touchPosition + ca.positionOffset)).length();
        if (a.incomingRetainState != kSS_Empty) {
            full = 0.0f;
            touchable = 1.0f;
        }
        float bumpy = full / touchable;
        bumpy = clampf_(bumpy - 0.001f, 0.0f, 1.0f);
        bumpy = curve(bumpy, 1.0f);
        bumpy = curve(bumpy, 0.5f);
        Vec3 curMom = w.m.ball.momentum;
        if (full < touchable && fabsf(desH - ball_predict(w.m.ball, 0).c[2]) < 1.0f) {
            float nba = nextBodyAngle();
            const int ft = ca.functionType;
            if (ft == kFtTrap || (ft == kFtBallControl && !pl.hasPossession)) {
                float xr = 0, yr = 0;
                Vec3 tv;
                if (!trap_vector(s, p, h.nextStartPosition, h.nextStartAngle.value(), nba,
                                 current_outgoing_movement(ca), ca, ca.frameNumber, h.spatial,
                                 h.decayingPositionOffset, xr, yr, tv))
                    return false;
                if (ca.originatingCommand.modifier & 1) tv *= 1.35f;
                tv = tv * (1.0f - bumpy) + curMom * bumpy;
                ball_touch(s, tv);
                ball_set_rotation(w, xr, yr, 0, 0.5f * (1.0f - bumpy));
                if (!team_set_last_touch(s, p, d.touchType)) return false;
            } else if (ft == kFtBallControl) {
                float xr = 0, yr = 0;
                Vec3 tv;
                if (!ball_control_vector(s, p, h.nextStartPosition, h.nextStartAngle.value(), nba,
                                         current_outgoing_movement(ca), ca, ca.frameNumber, h.spatial, xr, yr, tv))
                    return false;
                if (ca.originatingCommand.modifier & 1) tv *= 1.35f;
                tv = tv * (1.0f - bumpy) + curMom * bumpy;
                ball_touch(s, tv);
                ball_set_rotation(w, xr, yr, 0, 0.6f * (1.0f - bumpy));
                if (!team_set_last_touch(s, p, d.touchType)) return false;
            } else if (ft == kFtInterfere) {
                float xr = 0, yr = 0;
                Vec3 tv;
                if (!trap_vector(s, p, h.nextStartPosition, h.nextStartAngle.value(), nba,
                                 current_outgoing_movement(ca), ca, ca.frameNumber, h.spatial,
                                 h.decayingPositionOffset, xr, yr, tv))
                    return false;
                tv = tv * 0.5f + (ball_predict(w.m.ball, 0).flat() - h.spatial.position).normalized() * 4.0f +
                     Vec3(0, 0, random_in_range(w.rng, 0.5f, 1.5f));
                tv = tv * (1.0f - bumpy) + curMom * bumpy;
                ball_touch(s, tv);
                // GRF passes the factor as the z rotation here (the bias stays 1).
                ball_set_rotation(w, xr, yr, 0.3f * (1.0f - bumpy));
                if (!team_set_last_touch(s, p, kTouchAccidental)) return false;
            } else if (ft == kFtSliding) {
                Vec3 tv = rot2d(d.ballDirection, h.spatial.angle.value());
                tv = tv * 6.0f + w.m.ball.momentum * -0.28f;
                tv += Vec3(0, 0, 6);
                tv = tv * (1.0f - bumpy) + curMom * bumpy;
                ball_touch(s, tv);
                if (!team_set_last_touch(s, p, kTouchAccidental)) return false;
            } else if (ft == kFtShortPass || ft == kFtLongPass || ft == kFtHighPass) {
                const TouchInfo &ti = ca.originatingCommand.touchInfo;
                Vec3 bdir = ti.desiredDirection;
                float bpow = ti.desiredPower;
                int target = ti.targetPlayer;
                Vec3 inDir = ti.inputDirection;
                if (external_active(w, p)) inDir = keyboard_direction(w, p);
                Vec3 tdir = bdir;
                float tpow = bpow;
                int ttarget = -1;
                get_pass(w, p, ca.originatingCommand.desiredFunctionType, inDir, ti.inputPower, ti.autoDirectionBias,
                         ti.autoPowerBias, tdir, tpow, ttarget, ti.forcedTargetPlayer);
                float maxDev = 0.15f * kPi;
                float adiff = angle2d_to(tdir.flat(), bdir.flat());
                if (fabsf(adiff) <= maxDev) {
                    bdir = tdir;
                    bpow = tpow;
                    target = ttarget;
                } else if (fabsf(adiff) < 2.0f * maxDev) {
                    float cd = clampf_(adiff, -maxDev, maxDev);
                    bdir = rot2d(bdir, cd);
                    if (ttarget != target) {
                        float rb = nclamp(fabsf(cd), 0.0f, fabsf(adiff));
                        bpow = bpow * (1.0f - rb) + tpow * rb;
                        target = ttarget;
                    } else {
                        bpow = tpow;
                    }
                }
                if (target >= 0 && !team_select_player(s, teamID, target)) return false;
                float zr = 0.0f;
                Vec3 tv = bdir * 36 * (bpow + 0.3f);
                {
                    tv = best_possible_touch(s, p, tv, ca.functionType);
                    float bta = angle2d_to(h.spatial.bodyDirectionVector, tv) / kPi;
                    if (fabsf(bta) > 0.5f) bta = (1.0f - fabsf(bta)) * sign_side(bta);
                    bta *= 2.0f;
                    float amount = bta * 0.25f;
                    if (ca.functionType == kFtHighPass) amount *= 0.2f;
                    rot2d_inplace(tv, amount * (0.4f + 0.6f * nclamp(tv.length(), 0.0f, 70.0f)));
                    zr = amount * -340;
                }
                tv = tv * (1.0f - bumpy) + curMom * bumpy;
                ball_touch(s, tv);
                float fwd = 3.5f;
                if (ca.functionType == kFtHighPass) fwd = -1.3f;
                float tl = clampf_(tv.length(), 0.0, 15.0);
                float xr = tv.normalized(Vec3(0)).c[1] * (tl * fwd);
                float yr = tv.normalized(Vec3(0)).c[0] * (tl * fwd);
                ball_set_rotation(w, xr, yr, zr, 0.9f * (1.0f - bumpy));
                if (!team_set_last_touch(s, p, d.touchType)) return false;
            } else if (ft == kFtShot) {
                const TouchInfo &ti = ca.originatingCommand.touchInfo;
                Vec3 inDir = ti.inputDirection;
                if (external_active(w, p)) inDir = keyboard_direction(w, p);
                (void)shot_direction(w, p, inDir, ti.autoDirectionBias);  // unused result, as GRF
                float xr = 0, yr = 0, zr = 0;
                Vec3 tv = shot_vector(s, p, ca, h.spatial, h.decayingPositionOffset, xr, yr, zr);
                tv = tv * (1.0f - bumpy) + curMom * bumpy;
                ball_touch(s, tv);
                ball_set_rotation(w, xr, yr, zr, 0.7f * (1.0f - bumpy));
                if (!team_set_last_touch(s, p, d.touchType)) return false;
            } else if (ft == kFtDeflect) {
                bool canRetain = true;
                if (d.outgoingRetainRawValue == kSS_Empty) canRetain = false;
                if (w.m.ballRetainer != -1) canRetain = false;
                float vd = nclamp((w.m.ball.momentum - h.spatial.movement).length(), 0.0f, 40.0f);
                float rd = 0.0f;
                int ltp = team_by_id(w, 1 - teamID).lastTouchPlayer;
                if (ltp >= 0)
                    rd = lm::lm_powf(
                        last_touch_bias(w, ltp, cvt_f_i32(1200 - statistic(s, p, kStPhysicalReaction) * 400)), 0.6f);
                if ((1.0f - vd) * (1.0f - rd) < 0.3f) canRetain = false;
                if (canRetain) {
                    w.m.ballRetainer = p;
                } else {
                    Vec3 cbm = w.m.ball.momentum.flat();
                    Vec3 pm = h.spatial.movement;
                    float lat = random_in_range(w.rng, -1, 1);
                    Vec3 tv = (-cbm * 0.1f + pm * 2.0f + Vec3(-team_side(w, teamID), 0, 0) * 4.0f + Vec3(0, lat, 0))
                                  .normalized(Vec3(0)) *
                              (cbm.length() * 0.3f + pm.length() * 2.5f);
                    tv.c[2] += 1.2f;
                    tv = tv * (1.0f - bumpy) + curMom * bumpy;
                    ball_touch(s, tv);
                    ball_set_rotation(w, 0, 0, 0, 0.2f * (1.0f - bumpy));
                }
                if (!team_set_last_touch(s, p, kTouchAccidental)) return false;
            }
        }
    }
    if (w.m.ballRetainer == p) {
        if ((ca.touchFrame <= ca.frameNumber && d.outgoingRetainRawValue != kSS_Empty) ||
            (ca.touchFrame > ca.frameNumber && a.incomingRetainState != kSS_Empty) ||
            (d.incomingRetainRawValue != kSS_Empty && d.outgoingRetainRawValue != kSS_Empty)) {
            int bp = -1;
            if (d.outgoingRetainRawValue != kSS_Empty) bp = d.outgoingRetainBodyPart;
            if (bp < 0 && d.incomingRetainRawValue != kSS_Empty) bp = d.incomingRetainBodyPart;
            if (bp < 0) return s.fail(kStatusUnsupported);
            const Skeleton &sk = s.ctx.skeletons[p];
            Xform xf[kNodes];
            derive_nodes(sk, h.nodes, xf);
            const Xform &node = xf[sk.nodeMap[bp]];
            ball_touch(s, Vec3(0));
            ball_set_rotation(w, 0, 0, 0, 1.0f);
            ball_set_position(w, node.position + node.rotation * Vec3(0, 0, -0.36f));
            if (!team_set_last_touch(s, p, kTouchNonKicked)) return false;
        } else {
            w.m.ballRetainer = -1;
        }
    }
    return true;
}

// One tick of a player's humanoid.
CB_HDNI bool humanoid_process(const Sim &s, int p) {
    Match &w = s.w;
    Player &pl = w.m.players[p];
    Humanoid &h = pl.base.humanoid;
    AnimationState &ca = h.anim;
    const int teamID = w.playerTeamID[p];
    const Team &team = team_by_id(w, teamID);
    const Ball &ball = w.m.ball;
    const int mi = mental_index(w, h.mentalImageTime);
    h.decayingPositionOffset *= 0.95f;
    if ((double)h.decayingPositionOffset.length() < 0.005) h.decayingPositionOffset = Vec3(0);
    h.decayingDifficultyFactor = clampf_(h.decayingDifficultyFactor - 0.002f, 0.0f, 1.0f);
    bool teamTouchedLast = w.m.lastTouchTeamID == teamID;
    h.mentalImageTime = teamTouchedLast ? 0 : reaction_time_ms(s, p);
    calc_spatial_state(s, h);
    h.spatial.positionOffsetMovement = Vec3(0);
    ca.frameNumber++;
    h.prevAnimFrameNumber++;
    {
        const Anim &a = s.A(ca.anim);
        if (ca.frameNumber == a.frameCount - 1 && h.interruptAnim == kIntNone) h.interruptAnim = kIntSwitch;
        bool mayRequeue = true;
        if (mayRequeue && h.interruptAnim != kIntNone) mayRequeue = false;
        if (mayRequeue) {
            bool fnp = false;
            float ad = ((h.spatial.position + h.spatial.movement * 0.1f) - ball_predict(ball, 100).flat()).length();
            uint64_t second = team_slot(w, teamID) == 1 ? 1 : 0;
            uint64_t t = w.m.actualTime_ms;
            if (w.m.designatedPossessionPlayer == p && ad < 3.0f) fnp = ((t + second * 10) % 20) == 0;
            else if (w.m.designatedPossessionPlayer == p) fnp = ((t + second * 10) % 30) == 0;
            else if (team.designatedTeamPossessionPlayer == p) fnp = ((t + second * 20) % 40) == 0;
            else if (ad < 5.0f) fnp = ((t + second * 20) % 50) == 0;
            else if (ad < 10.0f) fnp = ((t + second * 40) % 80) == 0;
            if (!fnp) mayRequeue = false;
        }
        if (mayRequeue) {
            float bd = (mental_ball(w, mi, 500).flat() - h.spatial.position).length();
            const bool pending = ca.frameNumber < ca.touchFrame;
            if (((ca.functionType == kFtMovement && !pl.hasPossession && bd < 16.0f) ||
                 (ca.functionType == kFtMovement && pl.hasPossession) ||
                 (ca.functionType == kFtTrap && pending) || (ca.functionType == kFtBallControl && pending)) &&
                (a.incomingSpecialState == kSS_Empty) && (a.outgoingSpecialState == kSS_Empty))
                mayRequeue = true;
            else
                mayRequeue = false;
        }
        if (mayRequeue) h.interruptAnim = kIntReQueue;
    }
    convoy_waypoint(way_player(team_slot(w, teamID), p, 1));
    if (!crew_assist(s, kJobInterrupt, p, h.interruptAnim != kIntNone)) return false;
    h.requeueDelayFrames = h.requeueDelayFrames - 1 > 0 ? h.requeueDelayFrames - 1 : 0;
    h.interruptAnim = kIntNone;
    const Anim &a = s.A(ca.anim);
    {
        float bdNow = (ball_predict(ball, 0).flat() - h.spatial.position).length();
        float bdFut = (ball_predict(ball, 200).flat() - (h.spatial.position + h.spatial.movement * 0.2f)).length();
        float ltb = last_touch_bias(w, p, 1500);
        float oltb = team_last_touch_bias(w, 1 - teamID, 240);
        if (p == w.m.designatedPossessionPlayer &&
            ((ltb <= 0.01f && oltb <= 0.01f && ca.functionType == kFtMovement && bdNow < 0.6f && bdFut > 0.65f &&
              bdFut > bdNow) ||
             (ltb <= 0.7f && pl.hasPossession && ca.functionType == kFtTrip && bdNow < 0.4f)) &&
            ball_predict(ball, 0).c[2] < 1.6f)
            pl.triggerControlledBallCollision = true;
    }
    bool ctrlColl = pl.triggerControlledBallCollision;
    if (ctrlColl) pl.triggerControlledBallCollision = false;
    const bool touches = (ctrlColl && ca.touchFrame == -1) || ca.touchFrame == ca.frameNumber || w.m.ballRetainer == p;
    convoy_waypoint(way_player(team_slot(w, teamID), p, 2));
    if (!crew_assist(s, kJobTouches, p | (ctrlColl ? 0x10000 : 0), touches)) return false;
    const int eff = a.frameCount - 1;
    if (ca.touchFrame != -1 && ca.frameNumber <= ca.touchFrame) {
        float v = lm::lm_cosf((ca.frameNumber / (float)(ca.touchFrame + 1) - 0.5f) * kPi * 2.0f) + 1.0f;
        v = v * 0.1f + 0.9f;
        h.spatial.actionSmuggleMovement = (ca.actionSmuggle / (float)(ca.touchFrame + 1)) * v * 100.0f;
        ca.actionSmuggleOffset += h.spatial.actionSmuggleMovement / 100.0f;
    } else {
        h.spatial.actionSmuggleMovement = Vec3(0);
    }
    if (ca.touchFrame == -1 && ca.frameNumber <= eff) {
        float v = lm::lm_cosf((ca.frameNumber / (float)(eff + 1) - 0.5f) * kPi * 2.0f) + 1.0f;
        v = v * 0.1f + 0.9f;
        h.spatial.movementSmuggleMovement = (ca.movementSmuggle / (float)(eff + 1)) * v * 100.0f;
        ca.movementSmuggleOffset += h.spatial.movementSmuggleMovement / 100.0f;
    } else {
        h.spatial.movementSmuggleMovement = Vec3(0);
    }
    const int beginRot = 16;
    int capFrames = beginRot < eff + 1 ? beginRot : eff + 1;
    float cfb = std_min(1.0f, (ca.frameNumber + 1) / (float)capFrames);
    float bfb = cfb, efb = cfb;
    if (ca.touchFrame != -1) {
        int capTouch = beginRot < ca.touchFrame + 1 ? beginRot : ca.touchFrame + 1;
        bfb = std_min(1.0f, (ca.frameNumber + 1) / (float)capTouch);
        if (ca.frameNumber > ca.touchFrame)
            efb = (ca.frameNumber - ca.touchFrame) / (float)(eff - ca.touchFrame);
        else
            efb = 0.0f;
    }
    set_radian(ca.rotationSmuggleOffset,
               ca.rotationSmuggle.begin.value() * (1.0f - bfb) + ca.rotationSmuggle.end.value() * efb);
    if (w.m.ballRetainer == p && formation(s, p).role == kRoleGK && w.m.inSetPiece == false && w.m.inPlay == true) {
        const int side = team_side(w, teamID);
        const Vec3 bn = ball_predict(w.m.ball, 0);
        if (bn.c[1] > 20.05f) offset_position(w, p, Vec3(0, clampf_(20.05f - bn.c[1], -0.5f, 0.5f), 0) * 0.3f);
        if (bn.c[1] < -20.05f) offset_position(w, p, Vec3(0, clampf_(-20.05f - bn.c[1], -0.5f, 0.5f), 0) * 0.3f);
        if (bn.c[0] * -side > -kPitchHalfL + 16.4f)
            offset_position(w, p,
                            Vec3(clampf_((-kPitchHalfL + 16.4f) - bn.c[0] * -side, -0.5f, 0.5f), 0, 0) * -side * 0.3f);
        if (bn.c[0] * -side < -kPitchHalfL + 0.1f)
            offset_position(w, p,
                            Vec3(clampf_((-kPitchHalfL + 0.1f) - bn.c[0] * -side, -0.5f, 0.5f), 0, 0) * -side * 0.4f);
    }
    h.applyBuffer.frameNumber = ca.frameNumber;
    if ((uint32_t)ca.positions.count > (uint32_t)ca.frameNumber) {
        h.applyBuffer.position = h.startPosition + ca.positions[ca.frameNumber] + ca.actionSmuggleOffset +
                                 ca.actionSmuggleSustainOffset + ca.movementSmuggleOffset;
        set_radian(h.applyBuffer.orientation, h.startAngle.value() + ca.rotationSmuggleOffset.value());
        h.applyBuffer.noPosition = true;
    } else {
        h.applyBuffer.position =
            h.startPosition + ca.actionSmuggleOffset + ca.actionSmuggleSustainOffset + ca.movementSmuggleOffset;
        h.applyBuffer.orientation = h.startAngle;
        h.applyBuffer.noPosition = false;
    }
    for (int i = 0; i < kBodyParts; i++) h.applyBuffer.offsets[i] = h.offsets[i];
    return true;
}

}  // namespace cb
