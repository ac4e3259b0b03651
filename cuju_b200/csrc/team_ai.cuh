// cuju-b200: team AI — tactics update, offside trap, danger ranking, attacking runs, dynamic
// roles (Hungarian assignment) and man marking.
//   cuju include/cuju/simulation/team_ai.h:23-530
#pragma once

#include "ai_ctrl.cuh"

namespace cb {

CB_HD void tactics_set(Tactics &t, int id, float v) {
    t.present |= 1u << id;
    t.value[id] = round_trip_six(v);
}
// Goals and last-minute possession are stored in processing order (team_ai.h:30-36).
CB_HD int goal_count(const Match &w, int teamID) { return w.m.goalCount[teamID == w.firstTeamID() ? 0 : 1]; }
CB_HD float possession_last_minute(const Match &w) {
    return w.firstTeamID() == 1 ? -w.m.possessionLastMinute : w.m.possessionLastMinute;
}

// The user tactics every team shares, in the alphabetical order of their names; id -1 marks the
// two dribble tactics, which the update skips (team_ai.h:39-64).
struct UserTactic {
    int id;
    float value, modifier;
};
constexpr int kUserTactics = 12;
CB_HD UserTactic user_tactic(int i) {
    switch (i) {
        case 0: return {-1, 0.72f, 0.0f};
        case 1: return {-1, 0.5f, 0.0f};
        case 2: return {kDefenseDepth, 0.3f, 0.1f};
        case 3: return {kDefenseMicroFocusStrength, 0.96f, 0.15f};
        case 4: return {kDefenseMidfieldFocus, 0.96f, 0.3f};
        case 5: return {kDefenseSideFocusStrength, 0.16f, 0.1f};
        case 6: return {kDefenseWidth, 0.7f, 0.1f};
        case 7: return {kOffenseDepth, 0.34f, 0.1f};
        case 8: return {kOffenseMicroFocusStrength, 0.92f, 0.15f};
        case 9: return {kOffenseMidfieldFocus, 0.88f, 0.3f};
        case 10: return {kOffenseSideFocusStrength, 0.88f, 0.1f};
        default: return {kOffenseWidth, 0.74f, 0.1f};
    }
}

/// team_ai.h:66 (TeamUpdateTactics).
CB_HDNI void team_update_tactics(Match &w, int teamID) {
    TeamAIState &ai = team_by_id(w, teamID).ai;
    const int goals = goal_count(w, teamID), oppGoals = goal_count(w, 1 - teamID);
    ai.liveTactics = ai.baseTactics;
    float goalF = clampf_((float)(0.5 + (double)((oppGoals - goals) * 0.25f)), 0.0f, 1.0f);
    float timeF = 0.5f + 0.5f * clampf_((float)w.m.matchTime_ms / 6300000.0f, 0.0f, 1.0f);
    float offBias = clampf_(0.5f + (goalF - 0.5f) * (timeF * 1.0f), 0.0f, 1.0f);
    float posF = possession_last_minute(w) / 60.0f;
    float recent = teamID == 0 ? (float)(0.5 - (double)(posF * 0.5f)) : (float)(0.5 + (double)(posF * 0.5f));
    ai.offensivenessBias = offBias * 0.5f + recent * 0.5f;
    for (int i = 0; i < kUserTactics; i++) {
        const UserTactic t = user_tactic(i);
        float mult = t.modifier == 0.0f ? 0.0f : round_trip_six(t.modifier);
        float off = round_trip_six(t.value);
        off = (off - 0.5f) * 2.0f * mult;
        float base = t.id < 0 ? -1.0f : tactic(ai.baseTactics, t.id, -1.0f);
        if (base >= 0.0f) tactics_set(ai.liveTactics, t.id, clampf_(base + off, 0.0f, 1.0f));
    }
}

/// team_ai.h:101-115 (SelectAttackingRunPlayer, TeamApplyAttackingRun).
CB_HD int select_attacking_run_player(const Sim &s, int teamID) {
    const int pp = team_by_id(s.w, teamID).designatedTeamPossessionPlayer;
    Vec3 focus = hum(s.w, pp).spatial.position + Vec3(-team_side(s.w, teamID) * 26.0f, 0, 0);
    return closest_player(s, teamID, focus, true, pp);
}
CB_HD void team_apply_attacking_run(const Sim &s, int teamID, int manualPlayer) {
    TeamAIState &ai = team_by_id(s.w, teamID).ai;
    ai.endApplyAttackingRun_ms = s.w.m.actualTime_ms + 4000;
    ai.attackingRunPlayer = manualPlayer >= 0 ? manualPlayer : select_attacking_run_player(s, teamID);
}

/// team_ai.h:117 (TeamAIProcess).
CB_HDNI bool team_ai_process(const Sim &s, int teamID) {
    Match &w = s.w;
    MatchState &m = w.m;
    Team &team = team_by_id(w, teamID);
    const Team &opp = team_by_id(w, 1 - teamID);
    TeamAIState &ai = team.ai;
    const int side = team_side(w, teamID);
    auto posOf = [&](int p) { return hum(w, p).spatial.position; };
    auto movOf = [&](int p) { return hum(w, p).spatial.movement; };
    if (m.actualTime_ms % 1000 == 0) team_update_tactics(w, teamID);
    ai.teamHasPossession = team.hasPossession;
    ai.teamHasUniquePossession = team_unique_possession(w, teamID);
    ai.oppTeamHasPossession = opp.hasPossession;
    ai.oppTeamHasUniquePossession = team_unique_possession(w, 1 - teamID);
    ai.teamHasBestPossession = m.bestPossessionTeam == team_slot(w, teamID);
    ai.teamPossessionAmount = team.teamPossessionAmount;
    ai.fadingTeamPossessionAmount = team.fadingTeamPossessionAmount;
    ai.timeNeededToGetToBall = team.timeNeededToGetToBall_ms;
    ai.oppTimeNeededToGetToBall = opp.timeNeededToGetToBall_ms;

    const float ob = ai.offensivenessBias;
    float startD = 30.0f + 20.0f * ob;
    float forceD = 6.0f;
    float deepest = (kPitchHalfL - startD) * side;
    float bx = ball_predict(m.ball, 0).c[0];
    bx *= side;
    float offX = 20.0f + 10.0f * (1.0f - ob);
    float stf = nclamp(bx, kPitchHalfL - startD - offX, kPitchHalfL - forceD);
    bx += offX * (1.0f - stf);
    bx *= side;
    if (bx * side > deepest * side) deepest = bx;
    if (ball_predict(m.ball, 700).c[0] * side > deepest * side) deepest = ball_predict(m.ball, 700).c[0];
    const int opp_pp = opp.designatedTeamPossessionPlayer;
    if (opp_pp < 0) return s.fail(kStatusUnsupported);
    float caution = 4.0f * side;
    if ((posOf(opp_pp).c[0] + movOf(opp_pp).c[0] * 0.15f + caution) * side > deepest * side)
        deepest = posOf(opp_pp).c[0] + movOf(opp_pp).c[0] * 0.1f + caution;
    float lineX = offside_line(w, mental_index(w, 0), teamID);
    float slack = 4.0f;
    if (lineX * side - slack > deepest * side) deepest = lineX - slack * side;
    ai.offsideTrapX = deepest;

    PlayerList players;
    active_players(players, w, 1 - teamID);
    Vec3 mdp = Vec3((float)(((double)kPitchHalfL - 2.0) * side), 0, 0);
    mdp = mdp * 0.8f + ball_predict(m.ball, 100).flat() * 0.2f;
    if (players.count > 16) return s.fail(kStatusUnsupported);
    OpponentInfo info[kTeamPlayers];
    int n = 0;
    for (int i = 0; i < players.count; i++) {
        const int p = players[i];
        OpponentInfo e;
        e.player = p;
        e.dangerFactor = (1.0f - nclamp((posOf(p) - mdp).length(), 0, kPitchHalfL * 2));
        e.dangerFactor *= 0.95f;
        if (p == opp.designatedTeamPossessionPlayer) e.dangerFactor += 0.05f;
        info[n++] = e;
    }
    // Insertion sort, descending, equal ratings in order (std::sort's small-range path).
    for (int nx = 1; nx < n; nx++) {
        OpponentInfo mv = info[nx];
        int slot = nx;
        while (slot > 0 && mv.dangerFactor > info[slot - 1].dangerFactor) {
            info[slot] = info[slot - 1];
            slot--;
        }
        info[slot] = mv;
    }
    ai.opponentInfo.count = n;
    for (int i = 0; i < n; i++) ai.opponentInfo.el[i] = info[i];

    if (m.actualTime_ms % 500 == 0 && ai.endApplyAttackingRun_ms <= m.actualTime_ms) {
        if (gamer_count_enabled(team) < 2 && m.bestPossessionTeam == team_slot(w, teamID)) {
            const float needed = 0.5f;
            int runner = select_attacking_run_player(s, teamID);
            if (runner >= 0) {
                float d = (posOf(runner) - posOf(team.designatedTeamPossessionPlayer)).length();
                float dr = lm::lm_powf(1.0f - nclamp(d, 0, 40), 0.5f);
                Vec3 spot = posOf(runner) * Vec3(1.0f, 0.8f, 0.0f) + Vec3(side * 10.0f, 0, 0);
                PlayerList opps;
                closest_players(opps, s, 1 - teamID, spot, false, 4);
                float dens = 1.0f;
                for (int i = 0; i < opps.count; i++) {
                    float od = (posOf(opps[i]) - spot).length();
                    float inv = lm::lm_powf(curve(1.0f - nclamp(od, 0, 15), 1.0f), 0.5f);
                    dens -= inv * 0.3f;
                }
                if (dr * dens >= needed) team_apply_attacking_run(s, teamID, -1);
            }
        }
    }
    if (m.actualTime_ms % 1500 == 0) {
        const int d = team.designatedTeamPossessionPlayer;
        ai.forwardSupportPlayer =
            closest_player(s, teamID, posOf(d) * Vec3(1.0f, 1.0f, 0.0f) + Vec3(-side * 1.5f, 0, 0), false, d);
    }
    return true;
}

// Hungarian assignment (libhungarian's algorithm, as GRF runs it): reduces `cost` (size x size,
// row-major) in place and returns the total, or -1 when the reduced costs do not prove the
// assignment optimal; `colOfRow` is written only on success. team_ai.h:250 (HungarianSolve).
constexpr int kHungN = kTeamPlayers;
CB_HDNI int hungarian_solve(int *cost, int size, int *colOfRow_out) {
    const int kInf = 0x7FFFFFFF;
    auto C = [&](int r, int c) -> int & { return cost[r * size + c]; };
    int colOfRow[kHungN], unchosen[kHungN], rowDec[kHungN], slackRow[kHungN], rowOfCol[kHungN],
        parent[kHungN], colInc[kHungN], slack[kHungN];
    for (int i = 0; i < size; i++)
        colOfRow[i] = unchosen[i] = rowDec[i] = slackRow[i] = rowOfCol[i] = parent[i] = colInc[i] = slack[i] = 0;
    int row = 0, col = 0, red, nUnchosen, qpos, unmatched, total = 0, other;
    for (col = 0; col < size; col++) {
        red = C(0, col);
        for (row = 1; row < size; row++)
            if (C(row, col) < red) red = C(row, col);
        total += red;
        if (red != 0)
            for (row = 0; row < size; row++) C(row, col) -= red;
    }
    nUnchosen = 0;
    for (col = 0; col < size; col++) {
        rowOfCol[col] = -1;
        parent[col] = -1;
        colInc[col] = 0;
        slack[col] = kInf;
    }
    for (row = 0; row < size; row++) {
        red = C(row, 0);
        for (col = 1; col < size; col++)
            if (C(row, col) < red) red = C(row, col);
        rowDec[row] = red;
        bool matched = false;
        for (col = 0; col < size; col++)
            if (red == C(row, col) && rowOfCol[col] < 0) {
                colOfRow[row] = col;
                rowOfCol[col] = row;
                matched = true;
                break;
            }
        if (!matched) {
            colOfRow[row] = -1;
            unchosen[nUnchosen++] = row;
        }
    }
    if (nUnchosen != 0) {
        unmatched = nUnchosen;
        // Each pass of the outer loop augments one path; size bounds the number of passes.
        for (int guard = 0; guard <= size; guard++) {
            qpos = 0;
            bool breakthrough = false;
            // Every pass without a breakthrough queues one more row: at most size passes.
            for (int pass = 0; !breakthrough; pass++) {
                if (pass > size + 1 || nUnchosen > size) return -1;
                while (qpos < nUnchosen && !breakthrough) {
                    row = unchosen[qpos];
                    red = rowDec[row];
                    for (col = 0; col < size; col++)
                        if (slack[col]) {
                            int delta = C(row, col) - red + colInc[col];
                            if (delta < slack[col]) {
                                if (delta == 0) {
                                    if (rowOfCol[col] < 0) {
                                        breakthrough = true;
                                        break;
                                    }
                                    slack[col] = 0;
                                    parent[col] = row;
                                    unchosen[nUnchosen++] = rowOfCol[col];
                                } else {
                                    slack[col] = delta;
                                    slackRow[col] = row;
                                }
                            }
                        }
                    if (!breakthrough) qpos++;
                }
                if (breakthrough) break;
                red = kInf;
                for (col = 0; col < size; col++)
                    if (slack[col] && slack[col] < red) red = slack[col];
                for (qpos = 0; qpos < nUnchosen; qpos++) rowDec[unchosen[qpos]] += red;
                for (col = 0; col < size; col++)
                    if (slack[col]) {
                        slack[col] -= red;
                        if (slack[col] == 0) {
                            row = slackRow[col];
                            if (rowOfCol[col] < 0) {
                                for (other = col + 1; other < size; other++)
                                    if (slack[other] == 0) colInc[other] += red;
                                breakthrough = true;
                                break;
                            } else {
                                parent[col] = row;
                                unchosen[nUnchosen++] = rowOfCol[col];
                            }
                        }
                    } else {
                        colInc[col] += red;
                    }
            }
            while (true) {
                other = colOfRow[row];
                colOfRow[row] = col;
                rowOfCol[col] = row;
                if (other < 0) break;
                row = parent[other];
                col = other;
            }
            if (--unmatched == 0) break;
            nUnchosen = 0;
            for (col = 0; col < size; col++) {
                parent[col] = -1;
                slack[col] = kInf;
            }
            for (row = 0; row < size; row++)
                if (colOfRow[row] < 0) unchosen[nUnchosen++] = row;
        }
        if (unmatched != 0) return -1;
    }
    for (row = 0; row < size; row++)
        for (col = 0; col < size; col++)
            if (C(row, col) < rowDec[row] - colInc[col]) return -1;
    for (row = 0; row < size; row++) {
        col = colOfRow[row];
        if (col < 0 || C(row, col) != rowDec[row] - colInc[col]) return -1;
    }
    row = 0;
    for (col = 0; col < size; col++)
        if (colInc[col]) row++;
    if (row > size) return -1;
    for (int i = 0; i < size; i++) colOfRow_out[i] = colOfRow[i];
    for (int i = 0; i < size; i++) total += rowDec[i];
    for (int i = 0; i < size; i++) total -= colInc[i];
    return total;
}

/// team_ai.h:385 (TeamCalculateDynamicRoles).
CB_HDNI bool team_dynamic_roles(const Sim &s, int teamID) {
    Match &w = s.w;
    PlayerList all;
    active_players(all, w, teamID);
    int players[kTeamPlayers];
    int n = 0;
    if (all.count > 0) {
        if (formation(s, all[0]).role != kRoleGK) return s.fail(kStatusUnsupported);
        for (int i = 1; i < all.count; i++) players[n++] = all[i];
    }
    Vec3 slots[kTeamPlayers];
    for (int i = 0; i < n; i++) slots[i] = team_adapted_formation_position(s, players[i], false);
    // The integer distance of every (player, slot) pair, computed once.
    int icost[kTeamPlayers * kTeamPlayers];
    crew_map<int>(
        n * n,
        [&](int k) {
            const int pi = k / n, si = k % n;
            const SpatialState &sp = hum(w, players[pi]).spatial;
            Vec3 pp = sp.position + sp.movement * 0.5f;
            float d = (pp - slots[si]).length();
            return cvt_f_i32(roundf(d * 10));
        },
        icost);
    int sorted[kTeamPlayers * kTeamPlayers];
    const int nn = n * n;
    for (int i = 0; i < nn; i++) sorted[i] = icost[i];
    for (int u = 1; u < nn; u++)
        for (int k = u; k > 0 && sorted[k] < sorted[k - 1]; k--) {
            int t = sorted[k];
            sorted[k] = sorted[k - 1];
            sorted[k - 1] = t;
        }
    for (int cutoff = n; cutoff < nn; cutoff += 5) {
        // A row is a formation slot, a column a player.
        int cost[kTeamPlayers * kTeamPlayers];
        for (int pi = 0; pi < n; pi++)
            for (int si = 0; si < n; si++) {
                int c = icost[pi * n + si];
                if (c >= sorted[cutoff]) c = 50000;
                cost[pi + si * n] = c;
            }
        int colOfRow[kTeamPlayers];
        int total = hungarian_solve(cost, n, colOfRow);
        // The size comparison is unsigned: below five entries `size - 5` wraps and never holds.
        if (total != -1 && (total < 50000 || (unsigned)cutoff >= (unsigned)nn - 5u)) {
            for (int pi = 0; pi < n; pi++)
                for (int si = 0; si < n; si++)
                    if (colOfRow[si] == pi) {
                        const StaticFormation &f = formation(s, players[si]);
                        FormationEntry &e = w.m.players[players[pi]].dynamicFormationEntry;
                        e.role = f.role;
                        e.position = f.position;
                        e.startPosition = f.startPosition;
                        e.lazy = f.lazy;
                        e.controllable = f.controllable;
                    }
            break;
        }
    }
    return true;
}

/// team_ai.h:454 (TeamCalculateMarkingQuality).
CB_HDNI float marking_quality(const Match &w, int teamID, int player, int opponent) {
    const int side = team_side(w, teamID);
    const SpatialState &ps = hum(w, player).spatial, &os = hum(w, opponent).spatial;
    Vec3 op = os.position + os.movement * 0.1f;
    Vec3 pp = ps.position + ps.movement * 0.1f;
    Vec3 goal = Vec3(kPitchHalfL * side, 0, 0);
    Vec3 toGoal = goal - pp;
    float len = clampf_(toGoal.length(), 4.0f, 14.0f);
    Vec3 tgd = toGoal.normalized(Vec3(side, 0, 0));
    Vec3 safety = -tgd * 0.5f;
    Line2 line(pp + safety + rot2d(tgd, (float)(-0.5 * (double)kPi)) * len,
               pp + safety + rot2d(tgd, (float)(0.5 * (double)kPi)) * len);
    bool right = ((line.b.c[0] - line.a.c[0]) * (op.c[1] - line.a.c[1]) -
                  (line.b.c[1] - line.a.c[1]) * (op.c[0] - line.a.c[0])) > 0;
    float lp = 0.0f;
    float fromLine = line.distance_to(op, lp);
    float adapted = fromLine;
    if (right) adapted = fabsf(fromLine - 2.0f);
    float fromF = lm::lm_powf(nclamp(adapted, 0.0f, 60.0f), 0.5f);
    float onF = lm::lm_powf(clampf_(fabsf(lp * 2.0f - 1.0f), 0.0f, 1.0f), 0.5f);
    float r = 1.0f;
    r -= fromF * 0.5f;
    r -= onF * 0.5f;
    r = clampf_(r, 0.0f, 1.0f);
    if (!right) r *= 0.6f;
    float od = (1.0f - nclamp((pp - op).length(), 0.0f, kPitchHalfL * 2.0f));
    return r * 0.8f + od * 0.2f;
}

/// team_ai.h:496 (TeamCalculateManMarking).
CB_HDNI void team_man_marking(const Sim &s, int teamID) {
    Match &w = s.w;
    const TeamAIState &ai = team_by_id(w, teamID).ai;
    PlayerList players;
    active_players(players, w, teamID);
    for (int i = 0; i < players.count; i++) w.m.players[players[i]].manMarking = -1;
    const int marked = std_min((int)ai.opponentInfo.count, 3);
    for (int rank = 0; rank < marked; rank++) {
        int best = -1, bestIdx = 0;
        float bestQ = -1.0f;
        const int oppP = ai.opponentInfo.el[rank].player;
        float q[kTeamPlayers];
        crew_map<float>(
            players.count,
            [&](int i) {
                return formation(s, players[i]).role == kRoleGK ? -2.0f : marking_quality(w, teamID, players[i], oppP);
            },
            q);
        for (int i = 0; i < players.count; i++) {
            if (formation(s, players[i]).role == kRoleGK) continue;
            if (q[i] > bestQ) {
                best = players[i];
                bestQ = q[i];
                bestIdx = i;
            }
        }
        if (best >= 0) {
            w.m.players[best].manMarking = oppP;
            players.erase_at(bestIdx);
        }
        if (players.count == 0) break;
    }
}

}  // namespace cb
