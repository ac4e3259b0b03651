// cuju-b200: one tick of a team and of the whole match, and the pose update that ends a tick.
//   cuju include/cuju/simulation/team_process.h:150-300 (PlayerProcess, TeamProcess)
//   cuju include/cuju/simulation/match_process.h:25-370 (MatchProcess, put buffers)
//   cuju include/cuju/animation/apply.h:336 (FetchPutBuffersBatch)
#pragma once

#include "referee.cuh"

namespace cb {

/// team_process.h:150 (PlayerProcess).
CB_HDNI bool player_process(const Sim &s, int p) {
    Match &w = s.w;
    MatchState &m = w.m;
    Player &pl = m.players[p];
    if (!pl.base.isActive) return true;
    pl.desiredTimeToBall_ms = (pl.desiredTimeToBall_ms - 10 < 0) ? 0 : pl.desiredTimeToBall_ms - 10;
    if (external_active(w, p) && !human_controller_process(s, p)) return false;
    eliza_process(s, p);
    if (m.inPlay) {
        if (m.actualTime_ms % 1000 == 0) {
            auto &ph = pl.base.positionHistoryPerSecond;
            if (ph.count >= 512) return s.fail(kStatusOverflow);
            ph.el[ph.count++] = pl.base.humanoid.spatial.position;
        }
        if (pl.hasPossession) pl.possessionDuration_ms += 10;
        else pl.possessionDuration_ms = 0;
        if ((m.actualTime_ms + (uint64_t)(s.ctx.staticData->stableID[p] * 10)) % 100 == 0) tactical_situation(w, p);
    }
    Vec3 before = pl.base.humanoid.spatial.position;
    if (!humanoid_process(s, p)) return false;
    if (m.inPlay) {
        Vec3 after = pl.base.humanoid.spatial.position;
        float d = (after - before).length();
        // The raw statistic, without difficulty and fatigue scaling.
        const float stamina = s.ctx.staticData->data[p].statistics[kStPhysicalStamina];
        pl.base.fatigueFactorInverse -=
            d * 0.00003f * (2.0f - stamina) * (1.0f / s.ctx.staticData->matchDurationFactor);
        pl.base.fatigueFactorInverse = clampf_(pl.base.fatigueFactorInverse, 0.01f, 1.0f);
    }
    if (pl.cards > 1 && pl.cardEffectiveTime_ms <= m.actualTime_ms && active_count(w, w.playerTeamID[p]) > 1)
        return player_send_off(s, p);
    return true;
}

/// team_process.h:196 (TeamProcess).
CB_HDNI bool team_process(const Sim &s, int teamID) {
    Match &w = s.w;
    MatchState &m = w.m;
    Team &team = team_by_id(w, teamID);
    const Team &opp = team_by_id(w, 1 - teamID);
    team.teamPossessionAmount =
        (float)(opp.timeNeededToGetToBall_ms + 1500) / (float)(team.timeNeededToGetToBall_ms + 1500);
    float tmp = team.fadingTeamPossessionAmount * 0.995f + clampf_(team.teamPossessionAmount, 0.5f, 1.5f) * 0.005f;
    team.fadingTeamPossessionAmount += clampf_(tmp - team.fadingTeamPossessionAmount, -0.005f, 0.005f);
    if (!m.inPlay || m.inSetPiece || m.ballRetainer != -1) {
        float amount;
        if (m.ballRetainer != -1) amount = (w.playerTeamID[m.ballRetainer] == teamID) ? 1.5f : 0.5f;
        else amount = (m.bestPossessionTeam == team_slot(w, teamID)) ? 1.5f : 0.5f;
        team.fadingTeamPossessionAmount = team.teamPossessionAmount = amount;
    }
    team_gamers_select_anyone(s, teamID);
    convoy_waypoint(way_team(team_slot(w, teamID)));
    if (m.inPlay && !m.inSetPiece) {
        if (!team_ai_process(s, teamID)) return false;
        uint64_t off = teamID == (1 - w.firstTeamID()) ? 200 : 0;
        if ((m.actualTime_ms + off) % 400 == 0 && !team_dynamic_roles(s, teamID)) return false;
        if ((m.actualTime_ms + off + 100) % 400 == 0) team_man_marking(s, teamID);
        if (*s.status) return false;
    }
    for (int p = 0; p < m.playerCount; p++) {
        convoy_waypoint(way_player(team_slot(w, teamID), p, 0));
        if (w.playerTeamID[p] == teamID && m.players[p].base.isActive && !player_process(s, p)) return false;
    }
    if (m.inPlay) {
        for (int g = 0; g < team.gamers.count; g++) {
            HumanGamer &gm = team.gamers.el[g];
            int sel = gm.selectedPlayer;
            int bpp = team_best_possession_player(w, teamID);
            const bool *b = gm.controller.keyboard.buttons;
            // Every button's previous state reads as released: a held switch is a fresh press.
            const bool sw = b[kBtnSwitch] &&
                            (!(sel == bpp && sel == team.designatedTeamPossessionPlayer) || team.teamPossessionAmount < 1.0f);
            if (sw && sel < 0) return s.fail(kStatusUnsupported);
            if (sw && !m.players[sel].hasUniquePossession) {
                int tgt = -1;
                const bool bestTeam = m.bestPossessionTeam == team_slot(w, teamID);
                if (m.players[team.designatedTeamPossessionPlayer].base.externalController < 0 && bestTeam) {
                    tgt = team.designatedTeamPossessionPlayer;
                } else if (m.players[bpp].base.externalController < 0 && bestTeam) {
                    tgt = bpp;
                } else {
                    tgt = best_switch_target(s, teamID);
                    if (tgt >= 0 && m.players[tgt].base.externalController >= 0) tgt = -1;
                }
                if (tgt == team_goalie(s, teamID)) tgt = -1;
                if (tgt >= 0 && formation(s, tgt).controllable) {
                    team.mainSelectedPlayer = tgt;
                    gamer_set_selected(w, global_gamer(w, teamID, g), tgt);
                }
            }
        }
    } else if (m.actualTime_ms >= 2000) {
        if (dynamic_player_selection(w))
            for (int g = 0; g < team.gamers.count; g++)
                if (team.gamers.el[g].selectedPlayer >= 0) gamer_set_selected(w, global_gamer(w, teamID, g), -1);
        team.mainSelectedPlayer = -1;
    }
    int dt = (int)m.players[team.designatedTeamPossessionPlayer].timeNeededToGetToBall_ms;
    int best = team_best_possession_player(w, teamID);
    int ot = opp.timeNeededToGetToBall_ms;
    if (team.designatedTeamPossessionPlayer != best) {
        int d = team.designatedTeamPossessionPlayer;
        int bt = (int)m.players[best].timeNeededToGetToBall_ms;
        float r = (float)(bt + 500) / (float)(dt + 500);
        if (m.players[best].hasPossession) r *= 0.5f;
        if (m.players[d].hasPossession) r /= 0.5f;
        if (external_active(w, best)) r *= 0.8f;
        if (external_active(w, d)) r /= 0.8f;
        if (!external_active(w, best) && dt < ot - 100) {
            r += 0.2f;
            r *= 1.2f;
        }
        if (r < 0.8f) team.designatedTeamPossessionPlayer = best;
    }
    return true;
}

/// match_process.h:26 (PushMentalImage): slot 0 holds the newest of at most three images.
CB_HDNI void push_mental_image(Match &w) {
    MatchState &m = w.m;
    const int n = m.mentalImages.count < 3 ? m.mentalImages.count + 1 : 3;
    for (int i = n - 1; i > 0; i--) {
        crew_copy(m.mentalImages.el[i], m.mentalImages.el[i - 1]);
        w.flags.mentalBallMirrored[i] = w.flags.mentalBallMirrored[i - 1];
    }
    MentalImage &im = m.mentalImages.el[0];
    crew_copy_words(reinterpret_cast<uint32_t *>(&im), nullptr, (int)(sizeof(MentalImage) / 4));
    im.timeStamp_ms = (uint32_t)m.actualTime_ms;
    im.maxDistanceDeviation = 2.5f;
    im.maxMovementDeviation = kWalkVel;
    for (int slot = 0; slot < 2; slot++) {
        const int teamID = slot == 0 ? w.firstTeamID() : 1 - w.firstTeamID();
        PlayerList ps;
        active_players(ps, w, teamID);
        for (int i = 0; i < ps.count; i++) {
            const int p = ps[i];
            const SpatialState &sp = hum(w, p).spatial;
            PlayerImage pi;
            memset(&pi, 0, sizeof(pi));
            pi.player = p;
            pi.position = sp.position;
            pi.directionVector = sp.directionVector;
            pi.velocity = sp.velocityCategory;
            pi.movement = sp.movement;
            pi.role = m.players[p].dynamicFormationEntry.role;
            im.players.el[im.players.count++] = pi;
        }
    }
    const int np = (int)(kPredictionSpan_ms / 10);
    im.ballPredictions.count = np;
    crew_copy_words(reinterpret_cast<uint32_t *>(im.ballPredictions.el),
                   reinterpret_cast<const uint32_t *>(m.ball.predictions), np * 3);
    im.lazyFlip = m.ball.lazyFlip;
    w.flags.mentalBallMirrored[0] = false;
    m.mentalImages.count = n;
}

/// match_process.h:64 (CalculateBestPossessionTeamID).
CB_HD void best_possession_team(Match &w) {
    MatchState &m = w.m;
    if (m.ballRetainer != -1) {
        m.bestPossessionTeam = team_slot(w, w.playerTeamID[m.ballRetainer]);
        return;
    }
    const int first = w.firstTeamID();
    int ft = team_by_id(w, first).timeNeededToGetToBall_ms;
    int st = team_by_id(w, 1 - first).timeNeededToGetToBall_ms;
    if (ft < st) m.bestPossessionTeam = team_slot(w, first);
    else if (ft > st) m.bestPossessionTeam = team_slot(w, 1 - first);
    else m.bestPossessionTeam = -1;
}

/// match_process.h:82 (TriangleIntersectsLine); parameter bounds compare in double.
CB_HDNI bool triangle_intersects_line(const Vec3 *v, const Vec3 &normal, const Vec3 &ls, const Vec3 &le) {
    Vec3 e1 = v[1] - v[0];
    Vec3 e2 = v[2] - v[0];
    Vec3 d = le - ls;
    Vec3 so = ls - v[0];
    float num = -normal.dot(so);
    float den = normal.dot(d);
    if (fabsf(den) < 0.000001f) return false;
    float r = num / den;
    if ((double)r <= 0.0 || (double)r >= 1.0) return false;
    Vec3 iv = ls + d * r;
    float a11 = e1.dot(e1);
    float a12 = e1.dot(e2);
    float a22 = e2.dot(e2);
    Vec3 io = iv - v[0];
    float o1 = io.dot(e1);
    float o2 = io.dot(e2);
    float det = a12 * a12 - a11 * a22;
    float w1 = (a12 * o2 - a22 * o1) / det;
    if ((double)w1 < 0.0 || (double)w1 > 1.0) return false;
    float w2 = (a12 * o1 - a11 * o2) / det;
    if ((double)w2 < 0.0 || (double)(w1 + w2) > 1.0) return false;
    return true;
}

/// match_process.h:111 (CheckForGoal).
CB_HDNI bool check_for_goal(const Match &w, int side, const Vec3 &prev) {
    const Ball &b = w.m.ball;
    if ((double)fabsf(ball_predict(b, 10).c[0]) < (double)kPitchHalfL - 1.0) return false;
    const Vec3 ls = prev, le = ball_predict(b, 0);
    const float x = (kPitchHalfL + kLineHalfW + 0.11f) * side;
    const Vec3 normal(-side, 0, 0);
    const Vec3 lower[3] = {Vec3(x, 3.7f, 0), Vec3(x, -3.7f, 0), Vec3(x, 3.7f, 2.5f)};
    const Vec3 upper[3] = {Vec3(x, -3.7f, 0), Vec3(x, -3.7f, 2.5f), Vec3(x, 3.7f, 2.5f)};
    bool il = triangle_intersects_line(lower, normal, ls, le);
    bool iu = triangle_intersects_line(upper, normal, ls, le);
    if ((double)fabsf(prev.c[1]) > 3.7 && (double)fabsf(prev.c[0]) > (double)(kPitchHalfL - kLineHalfW) - 0.11)
        return false;
    return il || iu;
}

/// match_process.h:136 (MatchProcess). Returns false when the tick ends early (play waits for a
/// restart: only the clock advances) or on an unsupported path (status set).
CB_HDNI bool match_process(const Sim &s) {
    Match &w = s.w;
    MatchState &m = w.m;
    const bool rev = w.scenario.reverseTeamProcessing;
    const int first = w.firstTeamID(), second = 1 - first;

    convoy_waypoint(kWayBallCollisions);
    mirror_match(w, rev, !rev, rev);
    if (m.inPlay && !check_ball_collisions(s)) return false;
    if (!referee_process(s)) return false;
    Vec3 prevBall = ball_predict(m.ball, 0);
    mirror_match(w, rev, !rev, rev);
    if (!m.inPlay && m.referee.buffer.prepareTime + 10 < m.actualTime_ms) {
        bump_actual_time(s, 10);
        return false;
    }
    convoy_waypoint(kWayBallProcess);
    mirror_match(w, false, false, rev);
    ball_process(m.ball, m.ballIsInGoal);
    mirror_match(w, false, false, rev);

    convoy_waypoint(kWaySwitch);
    if (m.mentalImages.count == 0 || m.actualTime_ms % 100 == 0) push_mental_image(w);

    if (!team_update_switch(s, first)) return false;
    if (!team_update_switch(s, second)) return false;

    mirror_match(w, first == 1, first == 0, first == 1);
    if (!team_process(s, first)) return false;
    mirror_match(w, true, true, true);
    if (!team_process(s, second)) return false;
    mirror_match(w, first == 0, first == 1, first == 0);

    convoy_waypoint(kWayOfficials);
    mirror_match(w, rev, !rev, rev);
    if (!officials_process(s)) return false;
    mirror_match(w, rev, !rev, rev);

    convoy_waypoint(kWayPossession);
    mirror_match(w, first == 1, first == 0, first == 1);
    team_possession_stats(s, first);
    convoy_waypoint(kWayPossession + 1);
    mirror_match(w, true, true, true);
    team_possession_stats(s, second);
    mirror_match(w, first == 0, first == 1, first == 0);

    best_possession_team(w);
    if (m.ballRetainer == -1) {
        if (m.bestPossessionTeam != -1) {
            const int bt = m.bestPossessionTeam == 0 ? first : second;
            int cand = team_by_id(w, bt).designatedTeamPossessionPlayer;
            if (cand != m.designatedPossessionPlayer) {
                uint32_t dt = m.players[m.designatedPossessionPlayer].timeNeededToGetToBall_ms;
                uint32_t ct = m.players[cand].timeNeededToGetToBall_ms;
                float r = (float)(ct + 10) / (float)(dt + 10);
                if (r < 0.85f) m.designatedPossessionPlayer = cand;
            }
        } else {
            m.designatedPossessionPlayer =
                team_by_id(w, w.playerTeamID[m.designatedPossessionPlayer]).designatedTeamPossessionPlayer;
        }
    } else {
        m.designatedPossessionPlayer = m.ballRetainer;
    }

    convoy_waypoint(kWayCollisions);
    mirror_match(w, rev, !rev, rev);
    if (!check_humanoid_collisions(s)) return false;
    bump_actual_time(s, 10);
    bool g1 = false, g2 = false;
    if (m.inPlay) {
        g1 = check_for_goal(w, team_side(w, first), prevBall);
        g2 = check_for_goal(w, team_side(w, second), prevBall);
    }
    bool goal = g1 | g2;
    m.ballIsInGoal |= goal;
    mirror_match(w, rev, !rev, rev);
    if (m.inPlay) {
        if (goal) {
            // The ball entered one team's goal, so the other scores (goalCount in processing order).
            const int scorer = g1 ? second : first;
            m.goalCount[scorer == first ? 0 : 1] += 1;
            m.goalScored = true;
            m.lastGoalTeam = team_slot(w, scorer);
            team_update_tactics(w, scorer);
        }
        if (g1 || g2) {
            const int gt = m.lastGoalTeam == 0 ? first : second;
            bool own = true;
            if (m.lastTouchTeamIDs[kTouchKicked] == gt || m.lastTouchTeamIDs[kTouchNonKicked] == gt)
                own = false;
            m.lastGoalScorer = team_by_id(w, own ? 1 - gt : gt).lastTouchPlayer;
        }
    }
    if (m.inPlay && m.bestPossessionTeam != -1) {
        float sv = 0;
        sv += (team_by_id(w, 0).fadingTeamPossessionAmount - 0.5f) * team_side(w, 0);
        sv += (team_by_id(w, 1).fadingTeamPossessionAmount - 0.5f) * team_side(w, 1);
        auto &h = m.possessionSideHistory;
        if (h.count == 600) {
            // An overlapping shift: done serially (each lane the same values).
            for (int i = 0; i + 1 < h.count; i++) h.el[i] = h.el[i + 1];
            h.el[h.count - 1] = sv;
        } else {
            h.el[h.count++] = sv;
        }
    }
    Referee &ref = m.referee;
    if (ref.buffer.active && (ref.foul.foulType == 2 || ref.foul.foulType == 3) &&
        ref.buffer.stopTime < m.actualTime_ms - 1000) {
        auto set_auto = [&](bool a) {
            if (a != m.autoUpdateInGameCamera) {
                m.cameraPosition.count = 0;
                m.autoUpdateInGameCamera = a;
            }
        };
        if (ref.buffer.prepareTime > m.actualTime_ms) {
            set_auto(false);
            Vec3 rp = m.officials[0].humanoid.spatial.position;
            if (rev) rp.mirror();
            const Vec3 target = rp + Vec3(0, 0, 0.8f);
            const float zoom = 1.5f;
            m.cameraOrientation.set_angle_axis(0.4f * kPi, Vec3(1, 0, 0));
            m.cameraNodeOrientation.set_angle_axis((float)((double)angle2d(target) + 1.5 * (double)kPi), Vec3(0, 0, 1));
            m.cameraNodePosition = target - target.flat().normalized(Vec3(0, -1, 0)) * 10 * (1.0f / zoom) + Vec3(0, 0, 3);
            m.cameraFieldOfView = 60.0f;
            m.cameraNearCap = 1;
            m.cameraFarCap = 220;
            if (m.officials[0].humanoid.anim.functionType == kFtSpecial && m.referee.buffer.active) {
                m.referee.buffer.prepareTime = m.actualTime_ms + 1000;
                m.referee.buffer.startTime = m.referee.buffer.prepareTime + 2000;
            }
        } else {
            set_auto(true);
        }
    }
    return true;
}

/// match_process.h:285 (PlayerPreparePutBuffers); runs on one lane.
CB_HDNI void player_prepare_put_buffers(const Sim &s, int p) {
    Match &w = s.w;
    geometry_offsets(s, p);
    Player &pl = w.m.players[p];
    const Team &team = team_by_id(w, w.playerTeamID[p]);
    const bool ext = external_active(w, p);
    pl.bufferNameCaptionShowCondition = ext;
    int hg = 0;
    for (int g = 0; g < team.gamers.count; g++)
        if (!team.gamers.el[g].controller.keyboard.disabled) hg++;
    if (hg == 0) pl.bufferNameCaptionShowCondition = team.designatedTeamPossessionPlayer == p;
    int color = 5;
    const HumanGamer *gm = nullptr;
    if (pl.base.externalController >= 0) {
        const int ci = pl.base.externalController, n0 = w.m.teams[0].gamers.count;
        gm = ci < n0 ? &w.m.teams[0].gamers.el[ci] : &w.m.teams[1].gamers.el[ci - n0];
        color = gm->keyboardIndex % 6;
    }
    const float colors[6][3] = {{100, 140, 255}, {100, 255, 140}, {255, 110, 110},
                                {255, 255, 60},  {200, 80, 200},  {200, 200, 200}};
    pl.bufferPlayerColor = Vec3(colors[color][0], colors[color][1], colors[color][2]);
    if (ext && gm->controller.actionMode == 2)
        pl.bufferPlayerColor = pl.bufferPlayerColor * (lm::lm_sinf(w.m.actualTime_ms * 0.02f) * 0.3f + 0.7f);
}

/// match_process.h:323 (MatchPreparePutBuffers): lanes split a team; each player writes only its
/// own offsets and buffers.
CB_HDNI void match_prepare_put_buffers(const Sim &s) {
    Match &w = s.w;
    const int first = w.firstTeamID(), second = 1 - first;
    mirror_match(w, false, false, first == 1);
    {
        PlayerList ps;
        active_players(ps, w, first);
        crew_for(ps.count, [&](int i) { player_prepare_put_buffers(s, ps[i]); });
    }
    mirror_match(w, false, false, true);
    {
        PlayerList ps;
        active_players(ps, w, second);
        crew_for(ps.count, [&](int i) { player_prepare_put_buffers(s, ps[i]); });
    }
    mirror_match(w, false, false, first == 0);
}

/// match_process.h:344 + apply.h:336: every node of every humanoid in one split loop.
constexpr int kPutHumanoids = kPlayers + 3;
CB_HDNI bool match_fetch_put_buffers(const Sim &s) {
    Match &w = s.w;
    const int first = w.firstTeamID(), second = 1 - first;
    int16_t hidx[kPutHumanoids];
    int n = 0;
    for (int t = 0; t < 2; t++) {
        PlayerList ps;
        active_players(ps, w, t == 0 ? first : second);
        for (int i = 0; i < ps.count; i++) hidx[n++] = (int16_t)ps[i];
    }
    for (int o = 0; o < 3; o++) hidx[n++] = (int16_t)(w.m.playerCount + o);
    ApplyPlan plans[kPutHumanoids];
    int firstNode[kPutHumanoids + 1];
    firstNode[0] = 0;
    const AnimTables &T = s.T();
    for (int i = 0; i < n; i++) {
        Humanoid &h = any_hum(w, hidx[i]);
        const ApplyBuffer &b = h.applyBuffer;
        const Anim &a = T.anims[b.anim];
        if (!apply_prepare(T, a, h, b.smooth, b.frameNumber, plans[i])) return s.fail(kStatusOverflow);
        firstNode[i + 1] = firstNode[i] + a.nodeCount;
    }
    crew_sync();
    crew_for(firstNode[n], [&](int item) {
        int hi = 0;
        while (firstNode[hi + 1] <= item) hi++;
        Humanoid &h = any_hum(w, hidx[hi]);
        ApplyBuffer &b = h.applyBuffer;
        apply_node(T, T.anims[b.anim], s.ctx.skeletons[hidx[hi]], h, item - firstNode[hi], b.frameNumber, b.smooth,
                   b.smoothFactor, b.position, b.orientation.value(), b.offsets, 10, b.noPosition, plans[hi]);
    });
    return true;
}

/// match_process.h:362 (GameTaskProcessPhase): one 10 ms tick.
CB_HDNI bool game_tick(const Sim &s) {
    convoy_tick();
    bool process = match_process(s);
    if (*s.status) return false;
    convoy_waypoint(kWayCamera);
    update_camera(s);
    if (process) {
        convoy_waypoint(kWayPrepare);
        match_prepare_put_buffers(s);
        convoy_waypoint(kWayFetch);
        if (!match_fetch_put_buffers(s)) return false;
    }
    return *s.status == 0;
}

}  // namespace cb
