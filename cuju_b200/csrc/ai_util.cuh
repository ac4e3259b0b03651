// cuju-b200: helpers of the built-in player AI: mind sets, lines, formation positions adapted to
// the tactics and the ball, offside trap, situation ratings of a controller, the human
// controller's per-tick process, the closest-players ranking and the per-player tick.
//   cuju include/cuju/simulation/ai_controller.h:26-448
//   cuju include/cuju/simulation/player_controller.h:18-245
//   cuju include/cuju/simulation/team_process.h:23-188
#pragma once

#include "collisions.cuh"

namespace cb {

CB_HD float mind_set(int role) {
    float m = 0.5f;
    if (role == kRoleGK) m = 0.0f;
    if (role == kRoleCB) m = 0.0f;
    if (role == kRoleLB || role == kRoleRB) m = 0.25f;
    if (role == kRoleDM) m = 0.25f;
    if (role == kRoleLM || role == kRoleCM || role == kRoleRM) m = 0.5f;
    if (role == kRoleAM) m = 0.75f;
    if (role == kRoleCF) m = 1.0f;
    return m;
}
CB_HD float clamp_velocity(float v) {
    if (v < 0) return 0;
    if (v > kSprintVel) return kSprintVel;
    return v;
}

struct Line2 {
    Vec3 a, b;
    CB_HD Line2() {}
    CB_HD Line2(const Vec3 &s, const Vec3 &e) : a(s), b(e) {}
    CB_HD float closest(const Vec3 &p) const { return line_closest_to_point(a, b, p); }
    CB_HD float distance_to(const Vec3 &p, float &frac) const {
        frac = closest(p);
        Vec3 x;
        x.c[0] = a.c[0] + frac * (b.c[0] - a.c[0]);
        x.c[1] = a.c[1] + frac * (b.c[1] - a.c[1]);
        return (x - p).length();
    }
    CB_HD Vec3 intersection(const Line2 &l, float &frac) const {
        const Vec3 &s = l.a, &e = l.b;
        float div = (e.c[1] - s.c[1]) * (b.c[0] - a.c[0]) - (e.c[0] - s.c[0]) * (b.c[1] - a.c[1]);
        if (div == 0.0f) return a;
        frac = ((e.c[0] - s.c[0]) * (a.c[1] - s.c[1]) - (e.c[1] - s.c[1]) * (a.c[0] - s.c[0])) / (div);
        return a + (b - a) * frac;
    }
    CB_HD Vec3 intersection(const Line2 &l) const {
        float f = 0.0f;
        return intersection(l, f);
    }
};

CB_HD Vec3 clamped_2d(const Vec3 &self, const Vec3 &first, const Vec3 &second) {
    Vec3 r = self;
    float f2s = angle2d_to(second, first);
    int dir = sign_side(f2s);
    float f2self = angle2d_to(self, first);
    float s2self = angle2d_to(self, second);
    if (sign_side(f2self) != dir || sign_side(s2self) == dir) {
        if (fabsf(f2self) < fabsf(s2self)) r = first;
        else r = second;
    }
    return r;
}
CB_HDNI void quantize_direction(Vec3 &in, float bias) {
    Vec3 n = in.normalized(Vec3(0));
    const int dirs = 8;
    float a = angle2d(n);
    a /= kPi * 2.0f;
    a = roundf(a * dirs);
    a /= dirs;
    a *= kPi * 2.0f;
    in = (n * (1.0f - bias) + (rot2d(Vec3(1, 0, 0), a) * bias)).normalized(n) * in.length();
}
constexpr float kQuantizedDirBias = 0.0f;

CB_HD bool need_defending_movement(int mySide, const Vec3 &pos, const Vec3 &target) {
    float deep = std_max((target.c[0] - pos.c[0]) * -mySide, 0.0f);
    float wide = fabsf(target.c[1] - pos.c[1]);
    deep -= 0.5f;
    return wide > deep * 0.8f;
}
// A player missing from the mental image gets its first entry (GRF).
CB_HDNI PlayerImage mental_player_image(const Match &w, int mi, int p) {
    const MentalImage &im = w.m.mentalImages[mi];
    const int age = (int)(w.m.actualTime_ms - (uint64_t)im.timeStamp_ms);
    for (int i = 0; i < im.players.count; i++) {
        const PlayerImage &pi = im.players[i];
        if (pi.player != p) continue;
        PlayerImage n = pi;
        const SpatialState &sp = hum(w, pi.player).spatial;
        Vec3 extr = pi.movement * (float)age * 0.001f;
        n.position = pi.position + extr;
        n.position = n.position.max_deviation(sp.position, im.maxDistanceDeviation);
        n.movement = n.movement.max_deviation(sp.movement, im.maxMovementDeviation);
        return n;
    }
    return im.players[0];
}
CB_HDNI float player_average_velocity(const Match &w, int p, float period_s) {
    const auto &hist = w.m.players[p].base.positionHistoryPerSecond;
    unsigned int n = hist.count;
    if (n == 0) return 0;
    Vec3 prev;
    float total = 0;
    unsigned int c = 0;
    while (c <= (unsigned int)period_s) {
        Vec3 pos = hist[n - 1 - c];
        if (c > 0) total += (pos - prev).length();
        c++;
        if (n - c == 0) break;
        prev = pos;
    }
    return total / period_s;
}
CB_HD bool allow_last_ditch_p(const Match &w, int p, bool withPossession = true) {
    const Player &pl = w.m.players[p];
    if (withPossession && team_by_id(w, w.playerTeamID[p]).teamPossessionAmount < 1.0f) return true;
    return (float)pl.timeNeededToGetToBallOptimistic_ms * 1.7f + 800 < (float)pl.timeNeededToGetToBall_ms;
}
CB_HD float average_possession_side(const Match &w, unsigned int t_ms) {
    const auto &h = w.m.possessionSideHistory;
    float total = 0;
    unsigned int c = 0;
    for (int e = h.count - 1; e >= 0 && c <= t_ms / 10; e--) {
        total += h[e];
        c++;
    }
    if (c > 0) total /= (float)c;
    return total;
}
CB_HD float tactic(const Tactics &t, int id, float def = 0) { return ((t.present >> id) & 1) ? t.value[id] : def; }

constexpr float kDribbleOffensiveness = 0.5f;
constexpr float kDribbleCenterMagnet = 0.72f;

CB_HDNI float mixup(float base, int id, int role) {
    float v = -100.0f;
    if (role == kRoleCB) {
        if (id == kOffenseWidth) v = 0.2f;
    }
    if (role == kRoleLB || role == kRoleRB) {
        if (id == kDefenseOwnHalf) v = -0.075f;
        if (id == kOffenseWidth) v = 0.2f;
        if (id == kOffenseOwnHalf) v = -0.1f;
    }
    if (role == kRoleLM || role == kRoleRM) {
        if (id == kDefenseOwnHalf) v = -0.05f;
        if (id == kOffenseOwnHalf) v = -0.1f;
    }
    if (role == kRoleAM) {
        if (id == kDefenseDepth) v = 0.125f;
    }
    if (role == kRoleCF) {
        if (id == kDefenseDepth) v = 0.125f;
    }
    if (v > -100.0f) return clampf_(base + v, 0.0f, 1.0f);
    return base;
}

CB_HDNI Vec3 adapted_formation_position(const Sim &s, int p, float backX, float frontX, float lowY, float highY,
                                        float xFocus, float xFocusStrength, float yFocus, float yFocusStrength,
                                        const Vec3 &microFocus, float microFocusStrength, float midFocus,
                                        float midFocusStrength, bool useDynamic) {
    const Match &w = s.w;
    int side = team_side(w, w.playerTeamID[p]);
    Vec3 pos = useDynamic ? w.m.players[p].dynamicFormationEntry.position : formation(s, p).position;
    if (midFocusStrength > 0.0f) {
        float mpf = midFocus * 2.0f - 1.0f;
        float sb = clampf_(1.0f - fabsf(pos.c[0] * 1.2f), 0.0f, 1.0f);
        sb = curve(sb, 1.0f);
        sb *= midFocusStrength;
        pos.c[0] = pos.c[0] * (1.0f - sb) + mpf * sb;
    }
    float xl = frontX - backX;
    pos.c[0] = backX + (pos.c[0] * 0.5f + 0.5f) * xl;
    float yl = highY - lowY;
    pos.c[1] = lowY + (pos.c[1] * -side * 0.5f + 0.5f) * yl;
    Vec3 pure = pos;
    if (xFocusStrength > 0.0f) {
        float bias = 1.0f - clampf_(fabsf(xFocus - pos.c[0]) / fabsf(backX - frontX), 0.0f, 1.0f);
        bias = -lm::lm_cosf(bias * kPi) * 0.5f + 0.5f;
        bias = (float)lm::lm_pow((double)bias, 0.8);
        bias *= xFocusStrength;
        pos.c[0] = pos.c[0] * (1.0f - bias) + xFocus * bias;
    }
    if (yFocusStrength > 0.0f) {
        float d = clampf_(fabsf(yFocus - pos.c[1]) / fabsf(highY - lowY), 0.0f, 1.0f);
        float bias = 1.0f - d;
        bias *= 0.2f + 0.8f * fabsf(yFocus) / kPitchHalfW;
        bias *= yFocusStrength;
        pos.c[1] = pos.c[1] * (1.0f - bias) + yFocus * bias;
    }
    if (microFocusStrength > 0.0f) {
        float homY = 0.2f, homYPos = 0.4f;
        float sfd = ((microFocus - pure) * Vec3(1, 1.0f - homY, 0)).length() / 50.0f;
        float fd = sfd;
        if (fd < 1.0f) {
            float mfb = 1.0f;
            mfb *= 1.0f - fd;
            mfb = curve(mfb, 0.3f);
            float peakLoc = 0.15f, peakW = 0.25f, peakH = 0.1f;
            mfb += (1.0f - nclamp(fabsf(fd - peakLoc), 0.0f, peakW)) * peakH;
            mfb = clampf_(mfb, 0.0f, 1.0f);
            mfb *= microFocusStrength;
            Vec3 mfp = microFocus * Vec3(1, 1.0f - homYPos, 1) + pos * Vec3(0, homYPos, 0);
            pos = pos * (1.0f - mfb) + mfp * (mfb);
        }
    }
    return pos;
}

CB_HDNI Vec3 team_adapted_formation_position(const Sim &s, int p, bool useDynamic) {
    const Match &w = s.w;
    const int teamID = w.playerTeamID[p];
    const int side = team_side(w, teamID);
    const TeamAIState &ai = team_by_id(w, teamID).ai;
    const Tactics &tac = ai.liveTactics;
    const MatchState &m = w.m;
    int role = useDynamic ? m.players[p].dynamicFormationEntry.role : formation(s, p).role;
    Vec3 focal = hum(w, m.designatedPossessionPlayer).spatial.position;
    float urgency = 1.0f - nclamp((focal - hum(w, p).spatial.position).length(), 2.0f, 30.0f);
    float ballX = ball_average_position(w, cvt_f_u32(3500 * (1.0f - urgency * 0.7f))).c[0];
    float ballY = ball_average_position(w, cvt_f_u32(4000 * (1.0f - urgency * 0.5f))).c[1];
#define CB_TAC(id) mixup(tactic(tac, id), id, role)
    float offDepth = CB_TAC(kOffenseDepth), defDepth = CB_TAC(kDefenseDepth);
    float offWidth = CB_TAC(kOffenseWidth), defWidth = CB_TAC(kDefenseWidth);
    float offOwn = CB_TAC(kOffenseOwnHalf), defOwn = CB_TAC(kDefenseOwnHalf);
    float offMid = CB_TAC(kOffenseMidfieldFocus), defMid = CB_TAC(kDefenseMidfieldFocus);
    float offMidS = CB_TAC(kOffenseMidfieldFocusStrength), defMidS = CB_TAC(kDefenseMidfieldFocusStrength);
    float offSideS = CB_TAC(kOffenseSideFocusStrength), defSideS = CB_TAC(kDefenseSideFocusStrength);
    float offMicroS = CB_TAC(kOffenseMicroFocusStrength), defMicroS = CB_TAC(kDefenseMicroFocusStrength);
#undef CB_TAC
    const double mind = mind_set(role);
    offSideS = (float)((double)offSideS + (-0.5 + mind) * (double)0.2f);
    defSideS = (float)((double)defSideS + (0.5 - mind) * (double)0.2f);
    const float ob = ai.offensivenessBias;
    offSideS = clampf_(offSideS + -0.3f + (ob) * 0.3f, 0.0f, 1.0f);
    defSideS = clampf_(defSideS + -0.3f + (1.0f - ob) * 0.3f, 0.0f, 1.0f);
    float pab = nclamp(ai.fadingTeamPossessionAmount - 0.5f, 0.3f, 0.7f);
    float bb = nclamp(((ballX / kPitchHalfL) * -side), -0.7f, 0.7f);
    float bbb = 1.0f - fabsf(pab * 2.0f - 1.0f);
    bbb *= 0.6f;
    float pb = pab * (1.0f - bbb) + bb * bbb;
    pb = clampf_(pb + (ob - 0.5f) * 0.3f, 0.0f, 1.0f);
    focal = (ball_average_position(w, 3000).flat() * 1.0f + focal * 0.0f) * pb +
            (ball_average_position(w, 2000).flat() * 0.5f + focal * 0.5f) * (1.0f - pb);
    float depth = ai.depth * (offDepth * pb + defDepth * (1.0f - pb));
    float width = ai.width * (offWidth * pb + defWidth * (1.0f - pb));
    float offsetX = kPitchHalfL * side * ((offOwn * 2.0f - 1.0f) * pb + (defOwn * 2.0f - 1.0f) * (1.0f - pb));
    float sideS = (offSideS * pb + defSideS * (1.0f - pb));
    float sideFocus = pb * 2.0f - 1.0f;
    float sideX = 0.2f * sideFocus * -side * kPitchHalfL + 0.8f * -average_possession_side(w, 6000) * kPitchHalfL;
    float centerX = clampf_((ballX * (1.0f - sideS) + sideX * sideS) + offsetX, -kPitchHalfL, kPitchHalfL);
    float centerY = clampf_(ballY, -kPitchHalfW, kPitchHalfW);
    float fitD = 0.95f, fitW = 0.9f;
    centerX *= ((1.0f - depth) / 1.0f) * fitD + (1.0f - fitD);
    centerY *= ((1.0f - width) / 1.0f) * fitW + (1.0f - fitW);
    float backX = centerX - depth * kPitchHalfL * -side;
    float frontX = centerX + depth * kPitchHalfL * -side;
    float lowY = centerY - width * kPitchHalfW;
    float highY = centerY + width * kPitchHalfW;
    if (backX * side > ai.offsideTrapX * side) backX = clampf_(ai.offsideTrapX, -kPitchHalfL, kPitchHalfL);
    float yFocus = ballY * 1.0f;
    float yFocusS = 0.5f * pb + 0.2f * (1.0f - pb);
    Vec3 micro = focal;
    Vec3 defFocus = Vec3(clampf_(micro.c[0] + side * 2.0f, -kPitchHalfL, backX * side), micro.c[1] * 0.9f, 0);
    micro = (Vec3(clampf_(micro.c[0] - side * 1.0f, -kPitchHalfL, kPitchHalfL), micro.c[1] * 0.9f, 0)) * pb +
            (defFocus) * (1.0f - pb);
    float microS = (offMicroS * pb + defMicroS * (1.0f - pb));
    float msb = nclamp((ballX / kPitchHalfL) * -side, -0.7f, 0.7f);
    msb = msb * 0.7f + 0.3f;
    float autoMicro = (lm::lm_powf(msb, 0.8f) * pb + (lm::lm_powf(1.0f - msb, 0.6f)) * (1.0f - pb));
    microS = microS * (0.2f + 0.8f * autoMicro);
    float manualMid = (offMid * pb + defMid * (1.0f - pb));
    float autoMid = nclamp((ballX / kPitchHalfL) * -side, -0.8f, 0.8f);
    float midFocus = manualMid * 0.7f + autoMid * 0.3f;
    float midS = (offMidS * pb + defMidS * (1.0f - pb));
    Vec3 des = adapted_formation_position(s, p, backX, frontX, lowY, highY, 0.0f, 0.0f, yFocus, yFocusS, micro, microS,
                                          midFocus, midS, useDynamic);
    des.c[0] = clampf_(des.c[0], -kPitchHalfL, kPitchHalfL);
    des.c[1] = clampf_(des.c[1], -kPitchHalfW, kPitchHalfW);
    return des;
}

CB_HDNI void team_apply_offside_trap(const Match &w, int teamID, Vec3 &pos) {
    const int side = team_side(w, teamID);
    const float trapX = team_by_id(w, teamID).ai.offsideTrapX;
    float half = 2.0f;
    float ax = pos.c[0] * side;
    float at = trapX * side;
    if (ax > at - half) {
        float front = at - half;
        float fromFront = ax - front;
        float f = fromFront / (half * 2.0f);
        f = clampf_(f, 0.0f, 1.0f);
        float rx = front + half * f;
        pos.c[0] = rx * side;
    }
}

// ---------------------------------------------------------------------------------------------
// Player controllers (GRF PlayerController / ElizaController / HumanController).
CB_HD int base_reaction_time(const Sim &s, int p) {
    return cvt_f_i32(roundf(80.0f - statistic(s, p, kStPhysicalReaction) * 40.0f));
}
CB_HD int controller_reaction_time(const Sim &s, int p) {
    int rt = base_reaction_time(s, p);
    return cvt_f_i32((float)rt + (1.0f - team_difficulty(s.w, s.w.playerTeamID[p])) * 100);
}
// Before any touch the team processed first counts as the last to touch.
CB_HD int match_last_touch_player(const Match &w) {
    int teamID = w.m.lastTouchTeamID != -1 ? w.m.lastTouchTeamID : w.firstTeamID();
    return team_by_id(w, teamID).lastTouchPlayer;
}
CB_HD void eliza_process(const Sim &s, int p) {
    Player &pl = s.w.m.players[p];
    int rt = controller_reaction_time(s, p);
    if (match_last_touch_player(s.w) == p && pl.base.lastTouchType != kTouchAccidental) rt = 0;
    pl.base.controller.base.mentalImageTime = rt;
}
CB_HD ControllerState &active_controller(Match &w, int p) {
    if (external_active(w, p)) return gamer_of(w, p).controller.base;
    return w.m.players[p].base.controller.base;
}
CB_HDNI float free_space(const Match &w, int mi, int teamID, const Vec3 &focus, float safe, float future_s) {
    float cur = 0.0f;
    ImageList opp;
    mental_team_images(w, mi, 1 - teamID, opp);
    for (int i = 0; i < opp.count; i++) {
        ImagePos &o = opp[i];
        if (o.role == kRoleGK) continue;
        o.position = o.position + o.movement * 0.2f;
        Vec3 tfm = (focus - o.position).normalized(Vec3(0)) * kSprintVel * clampf_(future_s - 0.2f, 0.0f, 1000.0f);
        if (tfm.length() > (focus - o.position).length()) tfm = focus - o.position;
        o.position += tfm;
        float sit = 1.0f - clampf_((o.position - focus).length(), 0, safe) / safe;
        cur += sit;
    }
    return 1.0f - nclamp(cur, 0.0f, 2.5f);
}
CB_HDNI void tactical_situation(Match &w, int p) {
    Player &pl = w.m.players[p];
    const SpatialState &sp = pl.base.humanoid.spatial;
    const int teamID = w.playerTeamID[p];
    const int side = team_side(w, teamID);
    const int mi = mental_index(w, active_controller(w, p).mentalImageTime);
    float t = 0.5f;
    Vec3 check = sp.position + Vec3(-side, 0, 0) * kSprintVel * t;
    pl.tactical.forwardSpaceRating = free_space(w, mi, teamID, check, 5.0f, t);
    t = 0.1f;
    check = sp.position + sp.movement * t;
    pl.tactical.spaceRating = free_space(w, mi, teamID, check, 5.0f, t);
    pl.tactical.forwardRating =
        1.0f - clampf_((Vec3(kPitchHalfL * -side, 0, 0) - sp.position).length() / (kPitchHalfL * 2.0f), 0.0f, 1.0f);
    pl.tactical.forwardRating = lm::lm_powf(pl.tactical.forwardRating, 1.5f);
}
CB_HD bool team_unique_possession(const Match &w, int teamID) {
    return team_by_id(w, teamID).hasPossession && !team_by_id(w, 1 - teamID).hasPossession;
}
CB_HDNI void controller_situation(Match &w, int p, ControllerState &c) {
    const MatchState &m = w.m;
    const Player &pl = m.players[p];
    const int teamID = w.playerTeamID[p];
    const Team &t = team_by_id(w, teamID), &o = team_by_id(w, 1 - teamID);
    c.hasPossession = pl.hasPossession;
    c.hasUniquePossession = pl.hasUniquePossession;
    c.teamHasPossession = t.hasPossession;
    c.teamHasUniquePossession = team_unique_possession(w, teamID);
    c.oppTeamHasPossession = o.hasPossession;
    c.oppTeamHasUniquePossession = team_unique_possession(w, 1 - teamID);
    c.hasBestChanceOfPossession = t.designatedTeamPossessionPlayer == p;
    c.teamHasBestPossession = m.bestPossessionTeam == team_slot(w, teamID);
    c.possessionAmount = (float)(o.timeNeededToGetToBall_ms + 200) / (float)(c.timeNeeded_ms + 200);
    c.teamPossessionAmount = t.teamPossessionAmount;
    c.fadingTeamPossessionAmount = t.fadingTeamPossessionAmount;
    if (c.hasBestChanceOfPossession) {
        float d = nclamp((ball_predict(m.ball, 300).flat() - pl.base.humanoid.spatial.position).length(), 2.0f, 14.0f);
        float db = d * d;
        c.fadingTeamPossessionAmount = c.fadingTeamPossessionAmount * db + c.teamPossessionAmount * (1.0f - db);
    }
    c.oppTimeNeededToGetToBall = o.timeNeededToGetToBall_ms;
    c.hasBestPossession = c.hasPossession && c.possessionAmount >= 1.0f;
}

CB_HD void team_apply_attacking_run(const Sim &s, int teamID, int manualPlayer = -1);  // team_ai.cuh

CB_HDNI bool human_controller_process(const Sim &s, int p) {
    Match &w = s.w;
    MatchState &m = w.m;
    HumanControllerState &hc = gamer_of(w, p).controller;
    ControllerState &c = hc.base;
    const bool *b = hc.keyboard.buttons;
    int rt = base_reaction_time(s, p);
    if (match_last_touch_player(w) == p && m.players[p].base.lastTouchType != kTouchAccidental) rt = 0;
    c.mentalImageTime = rt;
    Vec3 cd;
    float unused = 0.0f;
    keyboard_input(w, p, cd, unused);
    hc.previousDirection = cd;
    hc.steadyDirection = cd;
    hc.lastSteadyDirectionSnapshotTime_ms = (int32_t)m.actualTime_ms;
    controller_situation(w, p, c);
    const int teamID = w.playerTeamID[p];
    const TeamAIState &ai = team_by_id(w, teamID).ai;
    if (hc.actionMode == 0 && (!m.inSetPiece || ai.taker == p)) {
        float pc = c.possessionAmount - 1.0f;
        if (m.designatedPossessionPlayer == p) {
            pc = 1.0f;
        } else {
            if (b[kBtnShortPass]) pc += 0.15f;
            if (b[kBtnLongPass]) pc += 0.15f;
            if (b[kBtnShot]) pc += 0.15f;
            if (b[kBtnPressure]) pc -= 0.15f;
            if (b[kBtnSliding]) pc -= 0.15f;
            if (b[kBtnTeamPressure]) pc -= 0.15f;
            if (ball_predict(m.ball, 0).c[2] > 1.5f) pc += 0.2f;
        }
        if (pc < 0.0f) {
            const bool allow = !m.inSetPiece;
            if (b[kBtnPressure] && allow) { hc.actionMode = 1; hc.actionButton = kBtnPressure; }
            if (b[kBtnSliding] && allow) { hc.actionMode = 1; hc.actionButton = kBtnSliding; }
            if (b[kBtnTeamPressure] && allow) { hc.actionMode = 1; hc.actionButton = kBtnTeamPressure; }
            if (b[kBtnKeeperRush] && allow) { hc.actionMode = 1; hc.actionButton = kBtnKeeperRush; }
        } else {
            bool allowHigh = true, allowShot = true;
            if (ai.taker == p && ai.setPieceType == kGmThrowIn) {
                allowHigh = false;
                allowShot = false;
            }
            if (b[kBtnShortPass]) { hc.actionMode = 2; hc.actionButton = kBtnShortPass; }
            if (b[kBtnLongPass]) { hc.actionMode = 2; hc.actionButton = kBtnLongPass; }
            if (b[kBtnHighPass] && allowHigh) { hc.actionMode = 2; hc.actionButton = kBtnHighPass; }
            if (b[kBtnShot] && allowShot) { hc.actionMode = 2; hc.actionButton = kBtnShot; }
        }
    }
    if (hc.actionMode == 2) {
        if (b[hc.actionButton]) {
            hc.gauge_ms += 10;
            hc.gauge_ms = (int)clampf_((float)hc.gauge_ms, 10, 1000);
            hc.actionBufferTime_ms = 0;
        } else {
            hc.actionBufferTime_ms += 10;
        }
    }
    if (b[kBtnSwitch] && c.hasPossession) team_apply_attacking_run(s, teamID);
    return true;
}

// ---------------------------------------------------------------------------------------------
CB_HD bool dynamic_player_selection(const Match &w) {
    const Scenario &sc = w.scenario;
    int l = 0, r = 0;
    for (int p = 0; p < sc.leftTeamSize; p++) l += sc.leftTeam[p].controllable ? 1 : 0;
    for (int p = 0; p < sc.rightTeamSize; p++) r += sc.rightTeam[p].controllable ? 1 : 0;
    return !((l == sc.leftAgents || sc.leftAgents == 0) && (r == sc.rightAgents || sc.rightAgents == 0));
}

// The `n` closest active players of a team into `r` (ties keep state order); distances in
// parallel. The list goes out through a reference: a list returned by value from a call that is
// not inlined, into a list declared inside a loop, was seen to share its stack slot with a live
// list of the caller in the sm_100a build.
CB_HDNI void closest_players(PlayerList &r, const Sim &s, int teamID, const Vec3 &pos, bool onlyAI,
                             unsigned int n = 3, bool onlySelectable = false) {
    const Match &w = s.w;
    float sd[kPlayers];
    int sp[kPlayers], count = 0;
    struct Cand {
        float distance;
        int32_t eligible;
    };
    auto eval = [&](int p) {
        Cand c{0.0f, 0};
        if (w.playerTeamID[p] != teamID || !w.m.players[p].base.isActive) return c;
        c.distance = (hum(w, p).spatial.position - pos).length();
        c.eligible = (!onlyAI || !external_active(w, p)) && (!onlySelectable || formation(s, p).controllable);
        return c;
    };
    crew_pipeline<Cand>(w.m.playerCount, eval, [&](int p, const Cand &c) {
        if (!c.eligible) return;
        const float d = c.distance;
        int slot = count++;
        for (; slot > 0 && d < sd[slot - 1]; slot--) {
            sd[slot] = sd[slot - 1];
            sp[slot] = sp[slot - 1];
        }
        sd[slot] = d;
        sp[slot] = p;
    });
    r.count = 0;
    for (unsigned int i = 0; i < n && (int)i < count; i++) r.push(sp[i]);
}

CB_HDNI int best_switch_target(const Sim &s, int teamID) {
    const Match &w = s.w;
    const MatchState &m = w.m;
    const Team &t = team_by_id(w, teamID);
    const int side = team_side(w, teamID);
    Vec3 action = hum(w, m.designatedPossessionPlayer).spatial.position * 0.5f + ball_predict(m.ball, 100).flat() * 0.5f;
    Vec3 def = (action * Vec3(1.0f, 0.8f, 0.0f)) + Vec3(side * 4.0f, 0.0f, 0.0f);
    Vec3 off = (action * Vec3(1.0f, 0.8f, 0.0f)) + Vec3(-side * 8.0f, 0.0f, 0.0f);
    def = def * 0.8f + hum(w, t.designatedTeamPossessionPlayer).spatial.position * 0.2f;
    float ob = t.fadingTeamPossessionAmount - 0.5f;
    ob = ob * 0.2f + clampf_(t.teamPossessionAmount - 0.5f, 0.0f, 1.0f) * 0.8f;
    ob = clampf_((float)((double)(ob - 0.5f) * 2.0 + 0.5), 0.0f, 1.0f);
    ob = clampf_(lm::lm_powf(ob, 1.5f), 0.0f, 1.0f);
    Vec3 res = def * (1.0f - ob) + off * ob;
    PlayerList tp;
    closest_players(tp, s, teamID, res, true, 8);
    PlayerList kept;
    for (int i = 0; i < tp.count; i++)
        if (formation(s, tp[i]).role != kRoleGK) kept.push(tp[i]);
    if (kept.count == 0) return -1;
    int best = 0;
    float late = 1.0f;
    int d = m.designatedPossessionPlayer;
    if (w.playerTeamID[d] != teamID) {
        const SpatialState &os = hum(w, d).spatial;
        Vec3 goal = Vec3(side * kPitchHalfL, 0.0f, 0.0f);
        float ogd = (goal - (os.position + os.movement * 0.5f)).length();
        for (int i = 0; i < kept.count; i++) {
            const SpatialState &ms = hum(w, kept[i]).spatial;
            float mgd = (goal - (ms.position + ms.movement * 0.5f)).length();
            if (mgd < ogd + late + clampf_(ogd * 0.1f, 0.0f, 3.0f)) {
                best = i;
                break;
            }
        }
    }
    return kept[best];
}

CB_HD int team_goalie(const Sim &s, int teamID) {
    const Match &w = s.w;
    for (int p = 0; p < w.m.playerCount; p++)
        if (w.playerTeamID[p] == teamID && w.m.players[p].base.isActive && formation(s, p).role == kRoleGK) return p;
    return -1;
}

}  // namespace cb
