// cuju-b200: the referee — half time, balls out of play, fouls, offside and set-piece starts.
//   cuju include/cuju/simulation/referee.h:20-350
#pragma once

#include "collisions.cuh"
#include "reset.cuh"

namespace cb {


/// referee.h:26 (BumpActualTime); `t` in milliseconds. Without referee animations the clock skips
/// the wait of a stoppage at once.
CB_HDNI void bump_actual_time(const Sim &s, uint64_t t) {
    MatchState &m = s.w.m;
    if (m.inPlay)
        m.matchTime_ms = (uint64_t)((float)m.matchTime_ms + t * (1.0f / s.ctx.staticData->matchDurationFactor));
    m.actualTime_ms += t;
    if (m.goalScored) m.goalScoredTimer += t;
    else m.goalScoredTimer = 0;
    if (m.inPlay && !m.inSetPiece) {
        const float sign = s.w.firstTeamID() == 1 ? -1.0f : 1.0f;
        float pos = m.possessionLastMinute * sign;
        int teamID = s.w.playerTeamID[m.designatedPossessionPlayer] == 0 ? 0 : 1;
        float delta = 0.001f * t;
        if (teamID == 0) {
            float mv = pos - delta, lim = -60.0f;
            pos = (mv < lim) ? lim : mv;
        } else {
            float mv = pos + delta, lim = 60.0f;
            pos = (lim < mv) ? lim : mv;
        }
        m.possessionLastMinute = pos * sign;
    }
}

/// referee.h:57 (MatchSetMatchPhase).
CB_HD void match_set_phase(Match &w, int phase) {
    w.m.matchPhase = phase;
    for (int p = 0; p < w.m.playerCount; p++) {
        PersonBase<AIControllerState> &b = w.m.players[p].base;
        if (!b.isActive) continue;
        b.fatigueFactorInverse += 1.0f;
        b.fatigueFactorInverse = clampf_(b.fatigueFactorInverse, 0.01f, 1.0f);
    }
}
/// Before any touch the first-processed team counts as the last to touch (referee.h:69).
CB_HD int match_last_touch_team(const Match &w) {
    return w.m.lastTouchTeamID != -1 ? w.m.lastTouchTeamID : w.firstTeamID();
}
CB_HD int static_side(int teamID) { return teamID == 0 ? -1 : 1; }
CB_HD void reset_foul(Foul &f) {
    f.foulPlayer = -1;
    f.foulType = 0;
    f.advantage = false;
    f.foulTime = 0;
    f.hasBeenProcessed = true;
}

/// referee.h:85 (RefereeStop).
CB_HDNI void referee_stop(const Sim &s, int setPiece, uint64_t extraPrepare = 0) {
    MatchState &m = s.w.m;
    RefereeBuffer &b = m.referee.buffer;
    m.inPlay = false;
    b.desiredSetPiece = setPiece;
    b.stopTime = m.actualTime_ms;
    b.prepareTime = m.actualTime_ms + 2000;
    bump_actual_time(s, 1900);
    if (extraPrepare) {
        b.prepareTime += extraPrepare;
        bump_actual_time(s, extraPrepare);
    }
    b.startTime = b.prepareTime + 2000;
}

/// referee.h:104 (RefereeCheckFoul); true when the foul stops play.
CB_HDNI bool referee_check_foul(const Sim &s) {
    Match &w = s.w;
    MatchState &m = w.m;
    Referee &ref = m.referee;
    Foul &f = ref.foul;
    bool penalty = false;
    if (f.foulType != 0) {
        if ((double)fabsf(f.foulPosition.c[1]) < 20.15 - (double)kLineHalfW &&
            (double)(f.foulPosition.c[0] * -static_side(w.playerTeamID[f.foulVictim])) >
                (double)kPitchHalfL - 16.5 + (double)kLineHalfW)
            penalty = true;
    }
    if (f.advantage) {
        if (penalty) {
            f.advantage = false;
        } else if (m.actualTime_ms - 600 > f.foulTime) {
            if (m.actualTime_ms - 3000 > f.foulTime) {
                f.foulPlayer = -1;
                f.foulType = 0;
            } else if (team_by_id(w, w.playerTeamID[f.foulVictim]).fadingTeamPossessionAmount < 1.0) {
                f.advantage = false;
            }
        }
    }
    if (f.foulType != 0 && f.advantage == false && !f.hasBeenProcessed) {
        RefereeBuffer &b = ref.buffer;
        const uint64_t extra = f.foulType >= 2 ? 10000 : 0;
        if (!penalty) {
            referee_stop(s, kGmFreeKick, extra);
            b.restartPosition = f.foulPosition;
        } else {
            referee_stop(s, kGmPenalty, extra);
            b.restartPosition =
                Vec3((float)(((double)kPitchHalfL - 11.0) * static_side(w.playerTeamID[f.foulPlayer])), 0, 0);
        }
        b.teamID = w.playerTeamID[f.foulVictim];
        b.active = true;
        Player &off = m.players[f.foulPlayer];
        if (f.foulType == 2) {
            off.cards++;
            off.cardEffectiveTime_ms = m.actualTime_ms + 6000;
        }
        if (f.foulType == 3) {
            off.cards += 3;
            off.cardEffectiveTime_ms = m.actualTime_ms + 6000;
        }
        f.hasBeenProcessed = true;
        return true;
    }
    return false;
}

/// referee.h:160 (RefereeProcess).
CB_HDNI bool referee_process(const Sim &s) {
    Match &w = s.w;
    MatchState &m = w.m;
    Referee &ref = m.referee;
    RefereeBuffer &b = ref.buffer;
    Foul &f = ref.foul;
    const Scenario &sc = w.scenario;
    if (m.inPlay && !m.inSetPiece) {
        Vec3 bp = ball_predict(m.ball, 0);
        // The half time is a wrapping int product compared with the unsigned match time.
        const int64_t half = (int32_t)((uint32_t)1800 * (uint32_t)sc.secondHalf);
        if (m.matchTime_ms >= (uint64_t)half && m.matchPhase == kPhaseFirstHalf) {
            m.inPlay = false;
            b.desiredSetPiece = kGmKickOff;
            b.stopTime = m.actualTime_ms;
            b.prepareTime = b.stopTime + 100;
            b.startTime = b.prepareTime + 200;
            b.restartPosition = sc.ballPosition;
            b.active = true;
            b.endPhase = true;
            b.teamID = left_team_owns_ball(w) ? 1 : 0;
            b.setPieceTeam = team_slot(w, b.teamID);
            b.taker = -1;
            reset_foul(f);
            match_set_phase(w, kPhaseSecondHalf);
        }
        if (sc.reverseTeamProcessing) bp.mirror();
        if ((double)fabsf(bp.c[0]) > (double)(kPitchHalfL + kLineHalfW) + 0.11 || m.goalScored) {
            f.advantage = false;
            bool isFoul = false;
            if (!m.goalScored) isFoul = referee_check_foul(s);
            else f.foulType = 0;
            if (!isFoul) {
                m.inPlay = false;
                const int ltt = match_last_touch_team(w);
                const int ls = static_side(ltt);
                if (m.goalScored) {
                    b.desiredSetPiece = kGmKickOff;
                    b.stopTime = m.actualTime_ms;
                    b.prepareTime = m.actualTime_ms + 500;
                    bump_actual_time(s, 400);
                    b.startTime = b.prepareTime + 500;
                    b.restartPosition = Vec3(0, 0, 0);
                    b.teamID = w.firstTeamID();
                    b.setPieceTeam = 1 - m.lastGoalTeam;
                } else if ((bp.c[0] > 0 && ls > 0) || (bp.c[0] < 0 && ls < 0)) {
                    referee_stop(s, kGmCorner);
                    float y = bp.c[1];
                    y = y > 0 ? kPitchHalfW : -kPitchHalfW;
                    b.restartPosition = Vec3(kPitchHalfL * ls, y, 0);
                    b.teamID = 1 - ltt;
                } else {
                    referee_stop(s, kGmGoalKick);
                    b.restartPosition = Vec3((float)((double)kPitchHalfL * 0.92 * -ls), 0, 0);
                    b.teamID = 1 - ltt;
                }
                b.active = true;
            }
        }
        if (ref.afterSetPieceRelaxTime_ms == 0) {
            if ((double)fabsf(bp.c[1]) > (double)(kPitchHalfW + kLineHalfW) + 0.11) {
                f.advantage = false;
                if (!referee_check_foul(s)) {
                    m.inPlay = false;
                    const int ltt = match_last_touch_team(w);
                    b.teamID = 1 - ltt;
                    referee_stop(s, kGmThrowIn);
                    b.restartPosition.c[0] = clampf_(bp.c[0], -kPitchHalfL + 0.6f, kPitchHalfL - 0.6f);
                    if (bp.c[1] > 0) b.restartPosition.c[1] = kPitchHalfW;
                    if (bp.c[1] <= 0) b.restartPosition.c[1] = -kPitchHalfW;
                    b.restartPosition.c[2] = 0;
                    b.active = true;
                }
            }
        }
        referee_check_foul(s);
    } else if (!m.inPlay && !m.inSetPiece && b.active == true) {
        if (b.prepareTime == m.actualTime_ms) {
            if (b.endPhase == true) {
                if (m.matchPhase == kPhasePreMatch) match_set_phase(w, kPhaseFirstHalf);
                b.endPhase = false;
            }
            MatchRng{w.rng}.seed(sc.gameEngineRandomSeed);
            if (!referee_prepare_set_piece(s, b.desiredSetPiece)) return false;
        }
        if (b.startTime == m.actualTime_ms) {
            m.inPlay = true;
            m.inSetPiece = true;
        }
    }
    if (m.inSetPiece) {
        bool taken = b.desiredSetPiece == kGmKickOff;
        if (!taken) {
            if (b.taker < 0) return s.fail(kStatusUnsupported);
            const AnimationState &ta = hum(w, b.taker).anim;
            taken = ta.touchFrame != -1 && !(ta.frameNumber < ta.touchFrame);
        }
        if (taken) {
            b.active = false;
            m.inSetPiece = false;
            team_by_id(w, 0).ai.setPieceType = kGmNormal;
            team_by_id(w, 1).ai.setPieceType = kGmNormal;
            ref.afterSetPieceRelaxTime_ms = 400;
            f.foulPlayer = -1;
            f.foulType = 0;
            if (m.matchPhase == kPhasePreMatch) match_set_phase(w, kPhaseFirstHalf);
        }
    }
    if (ref.afterSetPieceRelaxTime_ms > 0) ref.afterSetPieceRelaxTime_ms -= 10;
    return true;
}

/// referee.h:306 (RefereeBallTouched).
CB_HDNI bool referee_ball_touched(const Sim &s) {
    Match &w = s.w;
    MatchState &m = w.m;
    Referee &ref = m.referee;
    RefereeBuffer &b = ref.buffer;
    if (!w.scenario.offsides) return true;
    const int ltt = m.lastTouchTeamID;
    if (ltt == -1) return true;
    if (m.inPlay && !m.inSetPiece && b.active == false && active_count(w, 1 - ltt) > 1) {
        const int owner = match_last_touch_player(w);
        for (int i = 0; i < ref.offsidePlayers.count; i++) {
            if (ref.offsidePlayers.el[i] != owner) continue;
            ref.foul.advantage = false;
            if (!referee_check_foul(s)) {
                referee_stop(s, kGmFreeKick);
                b.restartPosition = pitch_position(w, owner);
                b.teamID = 1 - ltt;
                b.active = true;
            }
        }
    }
    ref.offsidePlayers.count = 0;
    if (m.inPlay && (b.active == false || (b.active == true && b.desiredSetPiece != kGmThrowIn &&
                                           b.desiredSetPiece != kGmCorner))) {
        // A fresh mental image: the defenders and the ball as they are this tick.
        ImageList im;
        PlayerList def;
        active_players(def, w, 1 - ltt);
        for (int i = 0; i < def.count; i++) {
            const SpatialState &sp = hum(w, def[i]).spatial;
            im.push(ImagePos{sp.position, sp.movement, m.players[def[i]].dynamicFormationEntry.role});
        }
        const int side = team_side(w, ltt);
        float line = offside_line_from_images(im, ball_predict(m.ball, 0), team_side(w, 1 - ltt), 0);
        const int tlp = team_by_id(w, ltt).lastTouchPlayer;
        PlayerList att;
        active_players(att, w, ltt);
        for (int i = 0; i < att.count; i++) {
            const int p = att[i];
            if (p == tlp) continue;
            if (hum(w, p).spatial.position.c[0] * side < line * side) {
                ref.offsidePlayers.el[ref.offsidePlayers.count++] = p;
            }
        }
    }
    return true;
}

}  // namespace cb
