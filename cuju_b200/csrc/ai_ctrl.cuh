// cuju-b200: the built-in player AI (GRF AIController): each tick it fills a player's command
// queue, in the order the animation selection tries them; the RNG draws happen in GRF's order.
//   cuju include/cuju/simulation/ai_controller.h:450-2230
#pragma once

#include "ai_util.cuh"

namespace cb {

struct AIController {
    const Sim &s;
    Match &w;
    const int player;
    MatchState &m;
    Player &pl;
    AIControllerState *eliza;  // null when an agent controls the player
    ControllerState &ctl;
    const int teamID, oppID, side;  // side: sign of the x coordinate of the own goal
    int mi = 0;                     // mental image index
    CommandQueue &q;

    CB_HD AIController(const Sim &sim, int p, CommandQueue &queue, ControllerState &c, AIControllerState *e)
        : s(sim), w(sim.w), player(p), m(sim.w.m), pl(sim.w.m.players[p]), eliza(e), ctl(c),
          teamID(sim.w.playerTeamID[p]), oppID(1 - sim.w.playerTeamID[p]),
          side(team_side(sim.w, sim.w.playerTeamID[p])), q(queue) {}

    CB_HD const SpatialState &SPo(int o) const { return hum(w, o).spatial; }
    CB_HD Vec3 pos(int o) const { return SPo(o).position; }
    CB_HD Vec3 mov(int o) const { return SPo(o).movement; }
    CB_HD Vec3 dir(int o) const { return SPo(o).directionVector; }
    CB_HD Vec3 pos() const { return pos(player); }
    CB_HD Vec3 mov() const { return mov(player); }
    CB_HD Vec3 dir() const { return dir(player); }
    CB_HD float float_velocity() const { return player_float_velocity(w, player); }
    CB_HD float stat(int k) const { return statistic(s, player, k); }
    CB_HD int static_role(int o) const { return formation(s, o).role; }
    CB_HD int dynamic_role() const { return pl.dynamicFormationEntry.role; }
    CB_HD const Team &team() const { return team_by_id(w, teamID); }
    CB_HD const Team &opp_team() const { return team_by_id(w, oppID); }
    CB_HD const TeamAIState &team_ai() const { return team().ai; }
    CB_HD Vec3 mball(int t) const { return mental_ball(w, mi, t); }
    CB_HD Vec3 ball(int t) const { return ball_predict(m.ball, t); }
    CB_HD float rnd(float lo, float hi) { return random_in_range(w.rng, lo, hi); }
    CB_HD void push(const PlayerCommand &c) { queue_push(s, q, c); }

    CB_HD float duel_likeliness() const {
        int o = opp_team().designatedTeamPossessionPlayer;
        Vec3 op = pos(o) + mov(o) * 0.1f;
        Vec3 meToOpp = op - (pos() + mov() * 0.1f);
        Vec3 oppToBall = mball(100).flat() - (pos(o) + mov(o) * 0.1f);
        float d = meToOpp.normalized(Vec3(0)).dot(oppToBall.normalized(Vec3(0)));
        d = d * 0.5f + 0.5f;
        return (1.0f - d);
    }

    CB_HDNI void add_defensive_component(Vec3 &desired, float bias, int forcedOpp = -1) const {
        int o = forcedOpp < 0 ? pl.manMarking : forcedOpp;
        if (!(m.inPlay && !m.inSetPiece && static_role(player) != kRoleGK)) return;
        if (o < 0) return;
        Vec3 defend = desired;
        float possShoot = 24.0f, genShoot = 8.0f;
        float minD = 0.4f, buf = 4.0f;
        PlayerImage oi = mental_player_image(w, mental_index(w, controller_reaction_time(s, player)), o);
        Vec3 op = oi.position + oi.movement * 0.5f;
        float thr = genShoot;
        if (o == m.designatedPossessionPlayer) thr = possShoot;
        Vec3 goal = Vec3(kPitchHalfL * side, 0, 0);
        float o2g = (goal - op).length();
        float o2t = clampf_(o2g - thr, minD, kPitchHalfL);
        Vec3 shoot = op + (goal - op).normalized(Vec3(0)) * o2t;
        const float trapX = team_ai().offsideTrapX;
        if (shoot.c[0] * side > trapX * side) {
            Line2 ogl(op, goal);
            Line2 offl(Vec3(trapX, -kPitchHalfW, 0), Vec3(trapX, kPitchHalfW, 0));
            shoot = ogl.intersection(offl);
            o2t = (shoot - op).length();
        }
        Vec3 meToThr = shoot - desired;
        float meToThrD = meToThr.length();
        float slack = meToThrD - (o2t - buf);
        if (slack > 0.0f) defend = desired + meToThr.normalized(Vec3(0)) * clampf_(slack, 0.0f, meToThrD);
        Vec3 actual = pos() + mov() * 0.14f;
        float a2t = (shoot - actual).length();
        float aslack = a2t - o2t;
        if (aslack > 0.0f) defend += (goal - defend).normalized(Vec3(0)) * aslack * 0.7f;
        desired = desired * (1.0f - bias) + defend * bias;
    }

    CB_HDNI Vec3 defend_position(int o, float distance = 0.0f) const {
        PlayerImage oi = mental_player_image(w, mi, o);
        Vec3 goal = Vec3(kPitchHalfL * side, 0, 0);
        Vec3 op = oi.position;
        Vec3 o2g = goal - op;
        Line2 ogl(op, goal);
        Line2 mol(pos(), op);
        Vec3 mid = mol.a * 0.5f + mol.b * 0.5f;
        Line2 perp(mid, mid + rot2d(mol.a - mid, (float)(0.5 * (double)kPi)));
        float frac = 0.0f;
        ogl.intersection(perp, frac);
        frac = clampf_(frac, 0.0f, 1.0f);
        Vec3 target = ogl.a + (ogl.b - ogl.a) * frac;
        target += (o2g.normalized(Vec3(0)) * kSprintVel * 0.1f) + (oi.movement * 0.14f) +
                  (o2g.normalized(Vec3(0)) * distance);
        return target;
    }

    CB_HDNI void keeper_deflect_command(bool onlyPickup) {
        if (static_role(player) != kRoleGK) return;
        if (get_distance(ball(400), pos()) > kBallDistOptimize + 10.0f) return;
        if (m.lastTouchTeamID == teamID && match_last_touch_player(w) != player &&
            m.lastTouchTeamIDs[kTouchKicked] == teamID)
            return;
        if (m.ballRetainer >= 0) return;
        if (fabsf(ball(160).c[1]) > 20.05f) return;
        if ((double)(ball(160).c[0] * -side) > -(double)kPitchHalfL + 16.4) return;
        PlayerCommand c;
        default_command(c);
        c.desiredFunctionType = kFtDeflect;
        c.useDesiredMovement = false;
        c.useDesiredLookAt = false;
        if (onlyPickup) c.onlyDeflectAnimationsThatPickupBall = true;
        push(c);
    }
    CB_HDNI void set_piece_command() {
        PlayerCommand c;
        default_command(c);
        c.desiredFunctionType = kFtMovement;
        c.useDesiredMovement = true;
        c.useDesiredLookAt = true;
        c.desiredDirection = dir();
        c.desiredVelocityFloat = kIdleVel;
        if (m.ballRetainer == player) c.desiredLookAt = pos() + ctl.inputDirection * 10.0f;
        else c.desiredLookAt = ball(0).flat();
        push(c);
    }
    CB_HDNI void ball_control_command(bool idleTurnToGoal = false, bool knockOn = false, bool stickyRun = false,
                                      bool keepBody = false) {
        if (get_distance(ball(200), pos()) > kBallDistOptimize) return;
        if (m.ballRetainer >= 0) return;
        if (!pl.hasPossession && !allow_last_ditch_p(w, player)) {
            float inv = 3.0f;
            if (fabsf(m.ball.momentum.c[2]) > 5.0f * inv) return;
            if ((m.ball.momentum.flat() - mov()).length() > 5.0f * inv) return;
        }
        if (m.designatedPossessionPlayer == player ||
            (team().designatedTeamPossessionPlayer == player && duel_likeliness() >= 0.25f)) {
            PlayerCommand c;
            default_command(c);
            c.desiredFunctionType = kFtBallControl;
            c.useDesiredMovement = true;
            c.desiredDirection = ctl.inputDirection;
            quantize_direction(c.desiredDirection, kQuantizedDirBias);
            c.desiredVelocityFloat = ctl.inputVelocityFloat;
            if (vel_category(c.desiredVelocityFloat) == kVelIdle && idleTurnToGoal) c.desiredDirection = Vec3(-side, 0, 0);
            if (knockOn) c.modifier |= 1;
            if (ctl.hasPossession && ctl.hasBestPossession && c.desiredVelocityFloat > kWalkSprintSwitch &&
                float_velocity() > kDribbleWalkSwitch && stickyRun) {
                float a = angle2d_to(c.desiredDirection, dir());
                if (fabsf(a) > 0.125f * kPi && fabsf(a) < 0.7f * kPi) {
                    if (a > 0) c.desiredDirection = rot2d(dir(), 0.125f * kPi);
                    if (a < 0) c.desiredDirection = rot2d(dir(), 0.125f * -kPi);
                }
            }
            c.useDesiredLookAt = true;
            const int vc = SPo(player).velocityCategory;
            if (keepBody && (vc == kVelWalk || vc == kVelDribble) && vel_category(c.desiredVelocityFloat) == kVelDribble) {
                c.desiredVelocityFloat = kWalkVel;
                c.desiredLookAt = pos() + dir() * 10.0f;
            } else {
                c.desiredLookAt = pos() + mov() * 0.2f + c.desiredDirection * 10.0f;
            }
            push(c);
        }
    }
    CB_HDNI void trap_command(bool idleTurnToGoal = false, bool knockOn = false) {
        if (m.ball.momentum.flat().length() < 2.0f) return;
        if (get_distance(ball(200), pos()) > kBallDistOptimize) return;
        if (m.ballRetainer >= 0) return;
        if (!ctl.hasPossession &&
            (m.designatedPossessionPlayer == player ||
             (team().designatedTeamPossessionPlayer == player && pl.timeNeededToGetToBallOptimistic_ms < 1000 &&
              ctl.oppTimeNeededToGetToBall > 400 && !ctl.oppTeamHasPossession && duel_likeliness() >= 0.5f))) {
            PlayerCommand c;
            default_command(c);
            c.desiredFunctionType = kFtTrap;
            c.useDesiredMovement = true;
            c.desiredDirection = ctl.inputDirection;
            quantize_direction(c.desiredDirection, kQuantizedDirBias);
            c.desiredVelocityFloat = ctl.inputVelocityFloat;
            if (static_role(player) == kRoleGK && !external_active(w, player)) {
                c.desiredDirection = Vec3(-side, 0, 0);
                c.desiredVelocityFloat = kIdleVel;
            }
            if (vel_category(c.desiredVelocityFloat) == kVelIdle && idleTurnToGoal) c.desiredDirection = Vec3(-side, 0, 0);
            if (knockOn) c.modifier |= 1;
            c.useDesiredLookAt = true;
            c.desiredLookAt = pos() + mov() * 0.3f + c.desiredDirection * 10.0f;
            push(c);
        }
    }
    CB_HDNI void interfere_command(bool byAnyMeans) {
        if (get_distance(ball(200), pos()) > kBallDistOptimize) return;
        if (m.ballRetainer >= 0) return;
        if (ctl.teamHasBestPossession) return;
        if (!byAnyMeans && duel_likeliness() < 0.2f) return;
        PlayerCommand c;
        default_command(c);
        c.desiredFunctionType = kFtInterfere;
        c.useDesiredMovement = true;
        c.strictMovement = byAnyMeans ? kStrictFalse : kStrictTrue;
        c.desiredDirection = ctl.inputDirection;
        c.desiredVelocityFloat = ctl.inputVelocityFloat;
        push(c);
    }
    CB_HDNI void sliding_command() {
        if (gamer_count_enabled(team()) != 0) return;
        if (m.ballRetainer >= 0) return;
        if (duel_likeliness() < 0.7f) return;
        if (!(!ctl.teamHasBestPossession && ctl.possessionAmount < 0.6f && m.designatedPossessionPlayer != player &&
              ctl.oppTeamHasPossession))
            return;
        const int o = ctl.opponentPlayer;
        Vec3 bp = mental_ball(w, mental_index(w, 20), 200);
        Vec3 pp = pos() + mov() * (float)0.2;
        float bd = (pp - bp).length();
        const AnimationState &oa = hum(w, o).anim;
        if ((bd > 0.7f && bd < 1.6f && ctl.oppTimeNeededToGetToBall > 260) ||
            (bd > 0.6f && bd < 1.8f && oa.functionType == kFtShot && oa.frameNumber < oa.touchFrame)) {
            PlayerCommand c;
            default_command(c);
            c.desiredFunctionType = kFtSliding;
            c.useDesiredMovement = true;
            c.desiredDirection = ((bp.flat() + mov(o) * 0.2f) - pp).normalized(Vec3(-side, 0, 0));
            c.desiredVelocityFloat = kSprintVel;
            c.useDesiredLookAt = true;
            c.desiredLookAt = pos() + mov() * 0.1f + c.desiredDirection * 10.0f;
            push(c);
        }
    }
    CB_HDNI unsigned int ball_control_movement(float desVel, Vec3 &bestDir, float &bestVel, Vec3 &bestLookAt) const {
        unsigned int desT = 250 + kTouchOffset_ms;
        Vec3 tbm = mball((int)desT).flat() - pos();
        float tbd = tbm.length();
        float adb = 1.0f;
        if (tbd < 0.4f) adb = lm::lm_powf(nclamp(tbd, 0.2f, 0.4f), 0.5f);
        Vec3 autoDir = tbm.normalized(dir());
        Vec3 manDir = dir();
        bestDir = autoDir * adb + manDir * (1.0f - adb);
        bestDir.normalize(dir());
        Vec3 bld = bestDir;
        bestVel = tbd * kDistToVel;
        // A velocity not below the dribble velocity, NaN included, takes the clamp.
        if (!(bestVel < kDribbleVel)) {
            bestVel = clampf_(desVel, bestVel, bestVel + 8.0f);
            if (range_velocity(bestVel) < bestVel) bestVel = bestVel * 0.9f + range_velocity(bestVel) * 0.1f;
            if (range_velocity(bestVel) > bestVel) bestVel = bestVel * 0.1f + range_velocity(bestVel) * 0.9f;
        }
        bestLookAt = pos() + bld * 10.0f;
        return pl.timeNeededToGetToBall_ms;
    }

    CB_HDNI unsigned int to_ball_movement(const Vec3 &desDir, float desVel, Vec3 &bestDir, float &bestVel,
                                          Vec3 &bestLookAt, float haste) const {
        const Vec3 pp = pos();
        const float maxV = max_velocity(*s.ctx.staticData, player);
        float movW = 1.0f, timeW = 0.0f, perpW = 0.1f, prevW = 0.0f;
        Vec3 ad = desDir;
        Line2 bl(mball(0).flat(), mball(1000).flat());
        float frac = 0;
        bl.distance_to(pp, frac);
        Vec3 shortest = bl.a + (bl.b - bl.a) * frac;
        Vec3 bsd = (mball(0).flat() - mball(1000).flat()).normalized(ad);
        float bsa = angle2d(bsd);
        Vec3 adbs = rot2d(ad, -bsa);
        const int dirs = 16;
        float a = angle2d(adbs);
        a /= kPi * 2.0f;
        a = roundf(a * dirs);
        a /= dirs;
        a *= kPi * 2.0f;
        float bias = 1.0f;
        adbs = (adbs * (1.0f - bias) + (rot2d(Vec3(1, 0, 0), a) * bias)).normalized(adbs);
        ad = rot2d(adbs, bsa);
        Vec3 desMov = ad * desVel;
        if (haste > 0.0f) {
            movW = 0.0f;
            timeW = 1.0f;
            perpW = 0.0f;
        }
        struct Choice {
            float rating = -10000.0f;
            int timeNeeded_ms = -10;
            int time_ms = -10;
        } best;
        const uint32_t ttb = pl.timeNeededToGetToBall_ms;
        unsigned int start = cvt_f_u32(clampf_((float)ttb, 40, (float)(kPredictionSpan_ms - 10)));
        Vec3 bpred = mball((int)start);
        if (fabsf(bpred.c[0]) > kPitchHalfL - 0.2f || fabsf(bpred.c[1]) > kPitchHalfW - 0.2f) start = 80;
        int prevDesired = pl.desiredTimeToBall_ms;
        int tnb = (int)ttb;
        Vec3 bmr = (mball((int)(ttb + 10)) - mball((int)ttb)).flat() * 100.0f;
        Vec3 bdr = bmr.normalized(ad);
        unsigned int step = 1;
        // The time needed at a grid time depends on that time alone, so a miss computes the next
        // 32 grid times across the lanes.
        uint32_t usual[32], optimistic[32];
        unsigned int firstCached = 0, cached = 0;
        auto time_at = [&](unsigned int qt) {
            if (qt < firstCached || qt >= firstCached + 10 * cached) {
                firstCached = qt;
                cached = crew_serial() ? 1 : (unsigned int)crew_width();
                uint64_t packed[32];
                crew_map<uint64_t>((int)cached,
                                  [&](int ln) {
                                      const unsigned int lt = qt + 10 * (unsigned int)ln;
                                      if (lt >= kPredictionSpan_ms) return (uint64_t)0;
                                      const Vec3 target = mball((int)lt).flat();
                                      TimeNeeded r = time_needed(pp, mov(), target, maxV, true, lt);
                                      return ((uint64_t)r.usual_ms << 32) | r.optimistic_ms;
                                  },
                                  packed);
                for (int ln = 0; ln < (int)cached; ln++) {
                    usual[ln] = (uint32_t)(packed[ln] >> 32);
                    optimistic[ln] = (uint32_t)packed[ln];
                }
            }
            TimeNeeded r;
            r.usual_ms = usual[(qt - firstCached) / 10];
            r.optimistic_ms = optimistic[(qt - firstCached) / 10];
            return r;
        };
        for (unsigned int t = start; t < kPredictionSpan_ms; t += 10 * step) {
            bool forced = false;
            Vec3 target = mball((int)t);
            if (fabsf(target.c[0]) > kPitchHalfL - 0.2f || fabsf(target.c[1]) > kPitchHalfW - 0.2f) forced = true;
            if (!forced)
                if (target.c[2] >= 1.0f) continue;
            target = target.flat();
            TimeNeeded tn = time_at(t);
            unsigned int tnm = tn.usual_ms;
            int ns = cvt_f_i32(roundf((float)(int)(tnm - t) * 0.05f)) - 5;
            ns = ns < 1 ? 1 : ns;
            ns = 10 < ns ? 10 : ns;
            step = (unsigned int)ns;
            if (tnm <= t) {
                float d = (target - pp).normalized(Vec3(0)).dot(bdr);
                float jit = clampf_((float)ttb / (float)t, 0.0f, 1.0f);
                if (jit < 0.35f) forced = true;
                if (d > 0.0f) forced = true;
                float td = (target - pp).length();
                float tv = clampf_(td * kDistToVel, kIdleVel, kSprintVel);
                Vec3 tm = (target - pp).normalized(Vec3(0)) * tv;
                float mr = 1.0f - nclamp((desMov - tm).length(), 0.0f, kSprintVel);
                float dr = 1.0f - nclamp(fabsf(angle2d_to(ad, tm.normalized(ad))), 0.0f, 0.5f * kPi);
                mr = mr * 0.4f + dr * 0.6f;
                float tr = 1.0f - nclamp((float)t, 0, 5000);
                float pr = 1.0f - nclamp((shortest - target).length(), 0, 2.0f * kSprintVel);
                float prevR = 0.0f;
                if (prevDesired >= tnb) {
                    int dd = prevDesired - tnb;
                    prevR = 1.0f - (dd < 0 ? -dd : dd) / 500.0f;
                }
                float rating = mr * movW + tr * timeW + pr * perpW + prevR * prevW;
                if (rating > best.rating || (forced && best.time_ms == -10)) {
                    best.rating = rating;
                    best.time_ms = (int)t;
                    best.timeNeeded_ms = (int)tnm;
                }
            }
            if (forced) {
                if (best.time_ms == -10) {
                    best.time_ms = (int)t;
                    best.timeNeeded_ms = (int)t;
                }
                break;
            }
        }
        if (best.time_ms == -10) {
            best.time_ms = kPredictionSpan_ms - 10;
            best.timeNeeded_ms = kPredictionSpan_ms - 10;
        }
        Vec3 target = mball(best.time_ms).flat();
        bestDir = (target - pp).normalized(dir());
        float bvt = clampf_(((float)best.timeNeeded_ms / (float)best.time_ms) * maxV, kIdleVel, kSprintVel);
        bestVel = bvt;
        if (best.time_ms > 250) bestVel = bestVel * 0.97f + float_velocity() * 0.03f;
        Vec3 lab = (mball(20).flat() - pp).normalized(ad);
        Vec3 lad = bestDir;
        Vec3 ladd;
        if (best.time_ms < 100) ladd = ad;
        else if (vel_category(bestVel) != kVelIdle) ladd = clamped_2d(ad, lab, lad);
        else ladd = ad;
        bestLookAt = pp + rot2d(lab, clampf_(angle2d_to(ladd, lab) * 1.0f, -0.25f * kPi, 0.25f * kPi)) * 10.0f;
        return (unsigned int)best.time_ms;
    }

    CB_HDNI void movement_command(bool forceMagnet, bool extraHaste) {
        const int lookT = 40;
        Vec3 qid = ctl.inputDirection;
        quantize_direction(qid, kQuantizedDirBias);
        PlayerCommand c;
        default_command(c);
        c.desiredFunctionType = kFtMovement;
        c.useDesiredMovement = true;
        c.useDesiredLookAt = true;
        Vec3 manDir = qid;
        float manVel = ctl.inputVelocityFloat;
        Vec3 defLook = manDir;
        float dvf = 1.0f - lm::lm_powf(nclamp(std_min(ctl.inputVelocityFloat, float_velocity()), kIdleDribbleSwitch,
                                              kSprintVel),
                                       0.5f) *
                               0.3f;
        Vec3 lfp = mball(lookT).flat();
        lfp += dir() * 0.5f;
        float tfa = angle2d_to((lfp - pos()).normalized(manDir), manDir);
        defLook = rot2d(manDir, tfa * lm::lm_powf(dvf, 0.7f));
        c.desiredDirection = manDir;
        c.desiredVelocityFloat = manVel;
        Vec3 autoDir = c.desiredDirection;
        float autoVel = c.desiredVelocityFloat;
        Vec3 autoLook = defLook;
        float apa = ctl.possessionAmount;
        pl.desiredTimeToBall_ms = 0;
        float autoBias = 0.0f;
        float ownHalf = nclamp(ctl.inputDirection.dot(Vec3(side, 0, 0)), -1.0f, 1.0f);
        const int td = team().designatedTeamPossessionPlayer;
        const float pa = ctl.possessionAmount;
        if (m.ballRetainer == player) {
            autoBias = 0.0f;
        } else if (forceMagnet || m.designatedPossessionPlayer == player ||
                   ((last_touch_bias(w, player, 2000) > 0.01f && pa > 0.5f) && td == player) ||
                   ((!ctl.oppTeamHasPossession && pa > 0.5f) && td == player) || (pa > 0.99f && td == player) ||
                   (ctl.hasBestPossession && td == player)) {
            if (ctl.hasBestPossession) {
                Vec3 al;
                pl.desiredTimeToBall_ms = (int)ball_control_movement(ctl.inputVelocityFloat, autoDir, autoVel, al);
                autoLook = (al - pos()).normalized(Vec3(0));
                autoBias = 1.0f;
            } else {
                float haste = 0.0f;
                if (extraHaste || forceMagnet) {
                    haste = 1.0f;
                } else {
                    float thr = 1.1f;
                    if (apa < thr) haste = 1.0f;
                }
                Vec3 al;
                pl.desiredTimeToBall_ms = (int)to_ball_movement(qid, ctl.inputVelocityFloat, autoDir, autoVel, al, haste);
                autoLook = (al - pos()).normalized(Vec3(0));
                autoBias = 1.0f;
                if (m.designatedPossessionPlayer != player) {
                    float sdf = 1.0f - clampf_(fabsf(angle2d_to(autoDir, manDir)) / kPi, 0.0f, 1.0f);
                    sdf = sdf * 0.5f + 0.5f;
                    autoBias = 0.0f;
                    if (last_touch_bias(w, player, 2000) > 0.01f) {
                        if (pl.timeNeededToGetToBall_ms < 1700)
                            autoBias = lm::lm_powf(last_touch_bias(w, player, 2000), 0.4f) * lm::lm_powf(sdf, 0.5f);
                    }
                    if (!ctl.oppTeamHasPossession) {
                        if (pl.base.externalController >= 0) {
                            float sb = last_switch_bias(w, ctl);
                            float mb = std_max(curve(sdf, 0.8f), lm::lm_powf(sb, 0.5f));
                            mb *= 1.0f - ownHalf;
                            autoBias = clampf_(lm::lm_powf((std_max(pa, 0.5f) - 0.5f) * 2.0f, 0.5f) * mb, autoBias, 1.0f);
                        }
                    }
                    if (forceMagnet) autoBias = 1.0f;
                }
            }
        } else if (w.playerTeamID[m.designatedPossessionPlayer] != teamID) {
            if (td == player) {
                PlayerImage oi = mental_player_image(w, mi, ctl.opponentPlayer);
                Vec3 op = oi.position + oi.movement * 0.14f + oi.directionVector * 0.6f;
                Vec3 o2g = (Vec3(kPitchHalfL * side, 0, 0) - op).normalized(Vec3(0));
                float ar = 5.0f;
                Vec3 fp = op + (o2g * ar * 0.7f);
                float actionBias = 1.0f - curve(nclamp((pos() - fp).length(), 0.0f, ar), 0.7f);
                if (external_active(w, player))
                    autoBias = actionBias * 0.0f + last_switch_bias(w, ctl) * 0.3f;
                else
                    autoBias = actionBias * 0.0f;
                autoBias *= 1.0f - ownHalf;
                if (autoBias > 0.0f) {
                    float pod = (op - pos()).length();
                    float mmb = lm::lm_powf(1.0f - curve(nclamp(pod, 0.0f, 7.0f), 0.7f), 1.2f);
                    Vec3 mmd = oi.movement.normalized(ctl.inputDirection);
                    float mmv = vel_float(oi.velocity);
                    Vec3 mml = (mball(lookT).flat() - pos()).normalized(Vec3(0));
                    Vec3 ht = op + o2g * pod * 0.3f;
                    Vec3 hm = ht - pos();
                    Vec3 hd = hm.normalized(ctl.inputDirection);
                    float hv = clampf_(hm.length() * kDistToVel, kIdleVel, kSprintVel);
                    Vec3 hl = (mball(lookT).flat() - pos()).normalized(Vec3(0));
                    autoDir = (mmd * mmb + hd * (1.0f - mmb)).normalized(ctl.inputDirection);
                    autoVel = clampf_(mmv * mmb + hv * (1.0f - mmb), kIdleVel, kSprintVel);
                    autoLook = ((mml * mmb + hl * (1.0f - mmb))).normalized(Vec3(0));
                }
            }
        }
        Vec3 am = autoDir * autoVel;
        Vec3 mm = manDir * manVel;
        Vec3 rm = mm * (1.0f - autoBias) + am * autoBias;
        c.desiredDirection = rm.normalized(qid);
        c.desiredVelocityFloat = clampf_(rm.length(), kIdleVel, kSprintVel);
        if (c.desiredVelocityFloat < kIdleDribbleSwitch) c.desiredDirection = autoLook;
        Vec3 rl = autoLook;
        c.desiredLookAt = pos() + rl * 10.0f;
        push(c);
    }

    CB_HDNI float lazy_velocity(float desVel) const {
        float a = desVel;
        if (a > kSprintVel) a = kSprintVel + (a - kSprintVel) * 0.1f;
        const float fi = pl.base.fatigueFactorInverse;
        float startL = 20.0f * (fi * 0.8f + 0.2f);
        float endL = 65.0f * (fi * 0.5f + 0.5f);
        Vec3 op = pos(opp_team().designatedTeamPossessionPlayer);
        float ad = (pos() - op).length();
        float tp = clampf_(ctl.fadingTeamPossessionAmount - 0.5f, 0.0f, 1.0f);
        float ms = mind_set(dynamic_role());
        float lr = ms + tp * (1.0f - ms * 2.0f);
        float lp = nclamp(ad, startL, endL);
        float lf = lp * (0.5f + lr * 0.5f);
        float r = a * (1.0f - lf);
        bool clampDribble = desVel >= kDribbleVel;
        if (clampDribble && r < kDribbleVel) r = kDribbleVel;
        float blf = 1.0f - nclamp(player_average_velocity(w, player, 10), kIdleVel, kSprintVel);
        float wr = stat(kStMentalWorkRate);
        blf = lm::lm_powf(blf, 0.8f - wr * 0.2f);
        blf = clampf_(blf * 1.2f, 0.0f, 1.0f);
        blf = blf * lf + 1.0f * (1.0f - lf);
        r = std_min(r, kSprintVel * blf);
        return r;
    }

    CB_HDNI Vec3 support_position_force_field(const Vec3 &base, bool makeRun) const {
        const int dp = team().designatedTeamPossessionPlayer;
        Vec3 cur = pos() + mov() * 0.1f;
        Vec3 mainMan = pos(dp) + mov(dp) * 0.1f;
        ForceField ff;
        float dms = mind_set(dynamic_role());
        bool noOffside = true;
        float baseW = 0.7f, overall = 1.0f;
        float oppRepel = 0.3f * overall, mateRepel = 0.4f * overall, ballRepel = 1.0f * overall, runW = 1.0f * overall,
              flock = 0.45f * overall;
        float web = 0.75f;
        switch (dynamic_role()) {
            case kRoleCB:
            case kRoleLB:
            case kRoleRB: oppRepel *= 2.2f; break;
            case kRoleDM: oppRepel *= 2.0f; break;
            case kRoleCM:
            case kRoleLM:
            case kRoleRM: oppRepel *= 1.6f; break;
            case kRoleAM: oppRepel *= 1.2f; break;
            case kRoleCF: oppRepel *= 1.0f; break;
            default: break;
        }
        float offX = offside_line(w, mi, oppID, 240);
        float amr = makeRun;
        {
            ForceSpot sp;
            sp.origin = base;
            if (player == team_ai().forwardSupportPlayer) {
                sp.origin.c[0] += -side * (0.3f + 0.7f * dms) * 12.0f;
            } else {
                float amount = 22.0f;
                float laneY = -sign_side(mainMan.c[1]) * 8.0f;
                amount *= curve(1.0f - nclamp(fabsf(laneY - cur.c[1]), 0.0f, 30.0f), 1.0f);
                float delta = -side * lm::lm_powf(dms, 1.5f) * amount;
                sp.origin.c[0] += delta;
            }
            sp.magnetType = kAttract;
            sp.decayType = kDecayConstant;
            sp.power = 1.0f * baseW;
            sp.power *= 0.3f + 0.7f * nclamp((sp.origin - cur).length(), 0.0f, 20.0f);
            field_push(s, ff, sp);
        }
        if (amr) {
            ForceSpot sp;
            sp.origin = Vec3(-side * kPitchHalfL, cur.c[1] * 0.5f, 0.0f);
            sp.magnetType = kAttract;
            sp.decayType = kDecayConstant;
            sp.power = 2.0f * runW;
            field_push(s, ff, sp);
        }
        PlayerList opps;
        closest_players(opps, s, oppID, mainMan * 0.3f + cur + 0.7f, false, 3);
        for (int i = 0; i < opps.count; i++) {
            PlayerImage oi = mental_player_image(w, mi, opps[i]);
            ForceSpot sp;
            Vec3 op = oi.position + oi.movement * 0.1f;
            sp.origin = op + (op - mainMan).normalized(Vec3(0)) * 2.0f;
            sp.magnetType = kRepel;
            sp.decayType = kDecayVariable;
            sp.power = 1.0f * oppRepel;
            sp.scale = 5.0f;
            if (amr) {
                sp.scale = 2.0f;
                sp.power *= 0.5f;
            }
            sp.exponent = 0.7f;
            field_push(s, ff, sp);
        }
        if (team().fadingTeamPossessionAmount >= 1.02f) {
            PlayerList mates;
            closest_players(mates, s, teamID, cur, false, 6);
            for (int i = 0; i < mates.count; i++) {
                if (mates[i] == player) continue;
                PlayerImage mimg = mental_player_image(w, mi, mates[i]);
                ForceSpot sp;
                sp.origin = mimg.position + mimg.movement * 0.1f;
                sp.magnetType = kRepel;
                sp.decayType = kDecayVariable;
                sp.power = 1.0f * mateRepel;
                sp.scale = 14.0f * web;
                sp.exponent = 1.0f;
                field_push(s, ff, sp);
            }
        }
        if (player != dp && team().fadingTeamPossessionAmount >= 1.06f) {
            ForceSpot sp;
            sp.magnetType = kRepel;
            sp.decayType = kDecayVariable;
            sp.power = 1.0f * ballRepel;
            sp.scale = 2.0f;
            sp.exponent = 0.5f;
            const int ts[4] = {200, 350, 500, 650};
            for (int i = 0; i < 4; i++) {
                sp.origin = mball(ts[i]).flat();
                field_push(s, ff, sp);
            }
        }
        if (player != dp) {
            ForceSpot sp;
            sp.origin = mainMan;
            sp.magnetType = kAttract;
            sp.decayType = kDecayVariable;
            sp.power = 1.0f * flock;
            sp.scale = 28.0f * web;
            sp.exponent = 1.0f;
            field_push(s, ff, sp);
            sp.magnetType = kRepel;
            sp.scale = 16.0f * web;
            field_push(s, ff, sp);
        }
        Vec3 ffp = cur + force_field_movement(ff, cur, 7);
        float margin = 0.08f;
        if (noOffside)
            if (ffp.c[0] * -side > (offX * -side) - margin) ffp.c[0] = offX - (margin * -side);
        ffp.c[0] = clampf_(ffp.c[0], -kPitchHalfL, kPitchHalfL);
        ffp.c[1] = clampf_(ffp.c[1], -kPitchHalfW, kPitchHalfW);
        return ffp;
    }

    enum StrategyKind { kDefense, kMidfield, kOffense };
    CB_HDNI void field_strategy_input(int kind, Vec3 &direction, float &velocity) const {
        const float staticFactor[3] = {1.0f, 0.9f, 0.8f};
        const float attackLow[3] = {0.2f, 0.1f, 0.1f}, attackHigh[3] = {0.9f, 0.7f, 0.6f};
        const float runThreshold[3] = {0.0f, 0.9f, 0.7f};
        const float defensiveBase[3] = {1.9f, 1.5f, 1.3f};
        Vec3 sdp = team_adapted_formation_position(s, player, false);
        Vec3 ddp = team_adapted_formation_position(s, player, true);
        float ad = nclamp(get_distance(pos(), pos(m.designatedPossessionPlayer)), 15.0f, 20.0f);
        float spb = curve(staticFactor[kind] * ad, 1.0f);
        Vec3 des = sdp * spb + ddp * (1.0f - spb);
        {
            float ab = nclamp((ctl.fadingTeamPossessionAmount - 0.5f) * 1.0f, attackLow[kind], attackHigh[kind]);
            bool makeRun = false;
            if (kind != kDefense && ab > runThreshold[kind]) {
                if (team_ai().endApplyAttackingRun_ms > m.actualTime_ms && team_ai().attackingRunPlayer == player)
                    makeRun = true;
            }
            Vec3 sup = support_position_force_field(des, makeRun);
            des = des * (1.0f - ab) + sup * ab;
        }
        {
            float ms = mind_set(dynamic_role());
            add_defensive_component(
                des, lm::lm_powf(clampf_(defensiveBase[kind] - ms - ctl.fadingTeamPossessionAmount, 0.0f, 1.0f), 0.7f));
            if (kind != kOffense) team_apply_offside_trap(w, teamID, des);
        }
        direction = (des - pos()).normalized(dir());
        float dv = (des - pos()).length() * kDistToVel;
        dv = lazy_velocity(dv);
        dv = clampf_(dv, 0, kSprintVel);
        velocity = dv;
    }

    CB_HDNI void ball_bound_for_goal() {
        eliza->ballBoundForGoal = false;
        bool intersect = false;
        eliza->ballBoundForGoalY = 0;
        float panic = 1.02f + (1.0f - (stat(kStMentalDefensivePositioning) * 0.6f + stat(kStMentalVision) * 0.4f)) * 0.5f;
        if (mball(4000).c[0] * side > kPitchHalfL && (pos() - mball(250)).length() < 32.0f) {
            Line2 b2g(mball(0).flat(), mball(800).flat());
            Line2 gl(Vec3(kPitchHalfL * side, -kPitchHalfW, 0), Vec3(kPitchHalfL * side, kPitchHalfW, 0));
            Vec3 ip = b2g.intersection(gl).flat();
            intersect = !((double)fabsf(ip.c[1]) > 3.7 * (double)panic);
            if (intersect) {
                eliza->ballBoundForGoalY = ip.c[1];
                eliza->ballBoundForGoal = true;
            }
        }
    }

    CB_HDNI void goalie_input(Vec3 &direction, float &velocity) {
        float lineDist = 10.0f;
        Vec3 bp = mball(cvt_f_i32(600 + (float)pl.timeNeededToGetToBall_ms * 0.2f)).flat();
        Vec3 target = Vec3((kPitchHalfL - lineDist) * side, 0, 0);
        Vec3 goal = Vec3(kPitchHalfL * side, 0, 0);
        float maxV = kSprintVel;
        if (bp.c[0] * side > 0) {
            ball_bound_for_goal();
            if (!eliza->ballBoundForGoal) {
                maxV = kSprintVel;
                Vec3 tfp = Vec3(kPitchHalfL * side, 3.7f, 0) - bp;
                Vec3 tsp = Vec3(kPitchHalfL * side, -3.7f, 0) - bp;
                float a = angle2d_to(tsp, tfp);
                Vec3 middle = rot2d(tfp, a * 0.5f).normalized(Vec3(side, 0, 0));
                Line2 b2g(bp, bp + middle);
                Line2 back(Vec3((kPitchHalfL - 0.7f) * side, -kPitchHalfW, 0), Vec3((kPitchHalfL - 0.7f) * side, kPitchHalfW, 0));
                Vec3 inter = b2g.intersection(back).flat();
                inter.c[1] = clampf_(inter.c[1], -3.7f, 3.7f);
                b2g.b = inter;
                float awayOff = 0.7f;
                float awayBias = 0.3f;
                awayBias *= nclamp(ctl.fadingTeamPossessionAmount, 1.0f, 1.5f);
                if (ctl.fadingTeamPossessionAmount < 1.0f) {
                    const int o = opp_team().designatedTeamPossessionPlayer;
                    Vec3 op = pos(o) + mov(o) * 0.32f;
                    if (m.players[o].hasPossession == false) b2g.a = op * 0.6f + bp * 0.4f;
                    else b2g.a = op * 0.4f + bp * 0.6f;
                    float st = 20.0f;
                    float o2g = (goal - op).length();
                    float o2t = clampf_(o2g - st * nclamp(o2g, 0.0f, st * 2.0f), 0.0f, kPitchHalfL);
                    Vec3 shoot = op + (goal - op).normalized(Vec3(0)) * o2t;
                    int mate = closest_player(s, teamID, shoot, false, player);
                    float m2t = 99999;
                    if (mate >= 0) {
                        Vec3 mp = pos(mate) + mov(mate) * 0.24f;
                        m2t = (shoot - mp).length();
                    }
                    if (m2t > o2t + 1.0f) {
                        awayBias = 1.0f;
                        int helper = closest_player(s, oppID, goal, false, o);
                        if (helper >= 0) {
                            Vec3 hp = pos(helper) + mov(helper) * 0.32f;
                            float hst = 24.0f;
                            float h2g = (goal - hp).length();
                            float h2t = clampf_(h2g - hst * nclamp(h2g, 0.0f, hst * 2.0f), 0.0f, kPitchHalfL);
                            Vec3 hshoot = hp + (goal - hp).normalized(Vec3(0)) * h2t;
                            int mh = closest_player(s, teamID, hshoot, false, player);
                            float mh2t = 99999;
                            if (mh >= 0) mh2t = (hshoot - (pos(mh) + mov(mh) * 0.24f)).length();
                            float sdd = 0.0f;
                            if (mh2t > h2t) sdd = nclamp(mh2t - h2t, 0.0f, 2.0f);
                            float hvp = 1.0f - nclamp(h2t / (o2t + 0.0001f), 1.0f, 1.5f);
                            hvp *= 0.7f;
                            awayBias = clampf_(1.0f - (sdd * hvp), 0.0f, 1.0f);
                        }
                    }
                }
                bool rush = team_ai().endApplyKeeperRush_ms > m.actualTime_ms;
                if (rush) awayBias = 1.0f;
                float d = std_max((b2g.a - b2g.b).length() - 0.5f, 0.0f);
                awayOff = clampf_(d * awayBias, awayOff, kPitchHalfL);
                target = b2g.b + (b2g.a - b2g.b).normalized(Vec3(0)) * awayOff;
                float frac = 0.0f;
                float dl = b2g.distance_to(pos(), frac);
                if ((target - goal).length() < (pos() - goal).length() && dl < 1.0f && frac > 0.0f) maxV = kWalkVel;
                target.c[0] = clampf_(target.c[0], -kPitchHalfL + 0.2f, kPitchHalfL - 0.2f);
            } else {
                maxV = kSprintVel;
                Line2 b2g;
                b2g.a = mball(10).flat();
                float minGL = 0.4f;
                Vec3 over = Vec3(kPitchHalfL * side, eliza->ballBoundForGoalY, 0);
                over += (b2g.a - over).normalized(Vec3(0)) * minGL;
                b2g.b = over;
                float frac = 0.0f;
                b2g.distance_to(pos() + mov() * 0.05f, frac);
                float frac1s = 0.0f;
                b2g.distance_to(mball(1010).flat(), frac1s);
                bool runsToGoal = false;
                if ((double)frac1s > 1e-4) {
                    float ttk = frac / frac1s;
                    Vec3 bak = mball(cvt_f_i32(10 + 1000 * ttk));
                    if ((double)bak.c[2] > 2.5) runsToGoal = true;
                }
                frac = clampf_(frac, 0.0f, 1.0f);
                if (runsToGoal) {
                    target = over;
                } else {
                    target = b2g.a + (b2g.b - b2g.a) * frac;
                    target.c[2] = 0.0f;
                    target.c[0] = clampf_(target.c[0], -kPitchHalfL + 0.2f, kPitchHalfL - 0.2f);
                }
            }
        }
        direction = target - pos();
        velocity = clampf_(direction.length() * kDistToVel, kIdleVel, maxV);
        direction.normalize(dir());
    }

    CB_HDNI float passing_odds(const Vec3 &target, int passType, const ImageList &opps, float bvm = 1.0f) const {
        float sec = 1.0f;
        Vec3 origin = pos() + mov() * 0.12f;
        Line2 line(origin, target);
        float danger = 0.0f;
        for (int i = 0; i < opps.count; i++) {
            Vec3 op = opps[i].position + opps[i].movement * 0.2f;
            float frac = 0.0f;
            float od = line.distance_to(op, frac);
            if (frac >= 0.0f && frac <= 1.0f + 0.2f) {
                if ((passType == kFtHighPass && (frac < 0.2f || frac > 0.65f)) || passType != kFtHighPass) {
                    float cf = clampf_(frac, 0.0f, 1.0f);
                    Vec3 inter = origin * (1.0f - cf) + target * cf;
                    float oti = (od + 1.0f) / kSprintVel;
                    Vec3 o2b = (inter - origin);
                    float pen = (passType == kFtHighPass && frac > 0.5f) ? 2.5f : 0.0f;
                    float bti = 0.7f + o2b.length() * frac * 0.03f + pen;
                    bti *= 1.0f / bvm;
                    danger += clampf_(bti - oti + (sec * 0.5f), 0.0f, sec);
                }
            }
        }
        if (passType == kFtHighPass) danger += 0.4f;
        danger = nclamp(danger, 0.0f, sec);
        return 1.0f - danger;
    }
    CB_HD float passing_odds_to(int target, int passType, const ImageList &opps) const {
        float itd = (pos(target) - pos()).length();
        if (passType == kFtHighPass && itd < 10.0f) return 0.0f;
        float est = 0.7f + itd * 0.03f;
        Vec3 tp = pos(target) + mov(target) * clampf_(est, 0.0f, 0.5f);
        if (passType == kFtLongPass) tp += Vec3(-side * itd * 0.2f, 0, 0);
        return passing_odds(tp, passType, opps);
    }
    CB_HDNI void add_pass(int target, int passType) {
        PlayerCommand c;
        default_command(c);
        c.desiredFunctionType = passType;
        c.useDesiredMovement = false;
        c.useDesiredLookAt = false;
        c.touchInfo.targetPlayer = -1;
        c.touchInfo.forcedTargetPlayer = target;
        c.touchInfo.inputDirection = Vec3(0);
        c.touchInfo.inputPower = 0;
        c.touchInfo.autoDirectionBias = 1.0f;
        c.touchInfo.autoPowerBias = 1.0f;
        TouchInfo &t = c.touchInfo;
        get_pass(w, player, passType, t.inputDirection, t.inputPower, t.autoDirectionBias, t.autoPowerBias,
                 t.desiredDirection, t.desiredPower, t.targetPlayer, t.forcedTargetPlayer);
        push(c);
    }
    CB_HDNI void add_panic_pass() {
        int ySide = sign_side(dir().c[1]);
        Vec3 away = ((dir() * Vec3(0.8f, 1.0f, 0.0f)).normalized() + Vec3(-side * 0.7f, ySide * 0.5f, 0))
                        .normalized(Vec3(0)) +
                    Vec3(0, 0, 0.3f);
        away.normalize(dir());
        PlayerCommand c;
        default_command(c);
        c.useDesiredMovement = false;
        c.useDesiredLookAt = false;
        c.touchInfo.inputDirection = away;
        c.touchInfo.desiredDirection = away;
        c.touchInfo.autoDirectionBias = 0.0f;
        c.touchInfo.autoPowerBias = 0.0f;
        c.desiredFunctionType = kFtHighPass;
        c.touchInfo.inputPower = 0.7f;
        c.touchInfo.desiredPower = 0.7f;
        push(c);
        c.desiredFunctionType = kFtShot;
        c.touchInfo.inputPower = 0.6f;
        c.touchInfo.desiredPower = 0.6f;
        push(c);
        c.desiredFunctionType = kFtLongPass;
        c.touchInfo.inputPower = 0.8f;
        c.touchInfo.desiredPower = 0.8f;
        push(c);
    }
    CB_HDNI void best_dribble_movement(Vec3 &desDir, float &desVel) const {
        Vec3 mp = pos(), mm = mov();
        float offF = 0.7f + kDribbleOffensiveness * 0.05f + mind_set(dynamic_role()) * 0.05f;
        float pm = 1.0f;
        float fut = 0.25f;
        PlayerList opps;
        closest_players(opps, s, oppID, mp, false, 5);
        List<PlayerImage, kPlayers> imgs;
        for (int i = 0; i < opps.count; i++) imgs.push(mental_player_image(w, mi, opps[i]));
        float nb = nclamp(fabsf(mp.c[0]) / kPitchHalfL, 0.0f, 1.0f);
        float cmi = 1.0f - nb * nb;
        cmi *= 0.5f;
        Vec3 og = Vec3(-side * kPitchHalfL, mp.c[1] * (1.0f - kDribbleCenterMagnet) * cmi, 0);
        ForceField ff;
        for (int i = 0; i < imgs.count; i++) {
            ForceSpot sp;
            sp.origin = imgs[i].position + imgs[i].movement * fut;
            sp.magnetType = kRepel;
            sp.decayType = kDecayVariable;
            sp.power = 2.0f * pm;
            sp.scale = 10.0f;
            sp.exponent = 1.0f;
            field_push(s, ff, sp);
        }
        {
            ForceSpot sp;
            sp.origin = Vec3(mp.c[0], (kPitchHalfW + 5.0f) * sign_side(mp.c[1]), 0);
            sp.magnetType = kRepel;
            sp.decayType = kDecayVariable;
            sp.power = 4.0f * pm;
            sp.scale = 20.0f;
            sp.exponent = 0.7f;
            field_push(s, ff, sp);
            sp.origin = Vec3((kPitchHalfL + 5.0f) * sign_side(mp.c[0]), mp.c[1], 0);
            field_push(s, ff, sp);
        }
        {
            ForceSpot sp;
            sp.origin = og;
            sp.magnetType = kAttract;
            sp.decayType = kDecayConstant;
            sp.power = offF * pm;
            field_push(s, ff, sp);
        }
        Vec3 ffm = force_field_movement(ff, mp + mm * fut, 1.0f);
        desDir = ffm.normalized(dir());
        desVel = clampf_(ffm.length() * kDistToVel, kIdleVel, kSprintVel);
        desVel = range_velocity(desVel);
    }

    CB_HDNI void on_the_ball_commands(Vec3 &rawDir, float &rawVel) {
        float md = nclamp((m.ball.momentum - mov()).length(), 0.0f, 10.0f);
        float oneTouchHard = md - stat(kStTechnicalShortPass) * md * 0.8f;
        ImageList oppImgs;
        mental_team_images(w, mi, oppID, oppImgs);
        float ptf = nclamp((float)pl.possessionDuration_ms, 0, 5000);
        float lpf = ptf * ptf;
        const float mind = mind_set(dynamic_role());
        float fsW = 0.4f, sW = 0.3f;
        float fW = 2.0f + mind * 6.0f;
        float totalTW = fsW + sW + fW;
        float tit = 0.06f * (1.0f - mind);
        float tdw = 1.0f + (mind * mind) * 10.0f;
        float passW = 1.0f;
        float passMin = 0.2f * (1.0f - mind) - lpf * 0.1f;
        float totalPW = tdw + passW;
        float passThr = 0.1f - lpf * 0.05f;
        const TacticalSituation &sit = pl.tactical;
        float tr = sit.forwardSpaceRating * fsW + sit.spaceRating * sW + sit.forwardRating * fW;
        tr /= totalTW;
        PlayerList mates;
        active_players(mates, w, teamID);
        float bestTotal = 0.0f;
        int bestP = -1;
        float bestPassR = 0.0f;
        int bestPassT = kFtShortPass;
        for (int i = 0; i < mates.count; i++) {
            const int mate = mates[i];
            if (mate == player) continue;
            const TacticalSituation &ms = m.players[mate].tactical;
            float mtr = ms.forwardSpaceRating * fsW + ms.spaceRating * sW + ms.forwardRating * fW;
            mtr /= totalTW;
            if (static_role(mate) == kRoleGK) mtr *= 0.7f;
            if (mtr > tr + tit) {
                float tdr = mtr - tr;
                float os = passing_odds_to(mate, kFtShortPass, oppImgs);
                float ol = passing_odds_to(mate, kFtLongPass, oppImgs);
                float oh = passing_odds_to(mate, kFtHighPass, oppImgs);
                float pr;
                int pt;
                if (os >= ol && os >= oh) {
                    pr = os;
                    pt = kFtShortPass;
                } else if (ol >= oh) {
                    pr = ol;
                    pt = kFtLongPass;
                } else {
                    pr = oh;
                    pt = kFtHighPass;
                }
                float total = tdr * tdw + pr * passW - oneTouchHard;
                total /= totalPW;
                if (total > bestTotal && total > passThr && pr > passMin) {
                    bestTotal = total;
                    bestP = mate;
                    bestPassR = pr;
                    bestPassT = pt;
                }
            }
        }
        if (mind < 0.25f) {
            float panicP = 1.0f - mind * 2.0f;
            float gc = 1.0f - nclamp((pos() - Vec3(kPitchHalfL * side, 0, 0)).length(), 2.0f, 16.0f);
            if (dynamic_role() != kRoleGK) {
                if ((bestP < 0 || bestPassR < panicP * gc) && ctl.possessionAmount < 0.9f + panicP * gc * 0.8f)
                    add_panic_pass();
            } else {
                if (ctl.possessionAmount < 3.0f) add_panic_pass();
            }
        }
        if (bestP >= 0) add_pass(bestP, bestPassT);
        float goalD = nclamp((Vec3(kPitchHalfL * -side, 0, 0) - pos()).length(), 0.0f, 32.0f);
        float ideal = 1.0f - nclamp((Vec3((kPitchHalfL - 7.0f) * -side, 0, 0) - pos()).length(), 0.0f, 16.0f);
        ideal = curve(ideal, 1.0f);
        if (ideal > 0.1f) {
            float lo = passing_odds(Vec3((kPitchHalfL + 1.0f) * -side, -3.6f, 0), kFtShot, oppImgs, 3.0f);
            float ce = passing_odds(Vec3((kPitchHalfL + 1.0f) * -side, 0.0f, 0), kFtShot, oppImgs, 3.0f);
            float hi = passing_odds(Vec3((kPitchHalfL + 1.0f) * -side, 3.6f, 0), kFtShot, oppImgs, 3.0f);
            float odds = ce, y = 0.0f;
            if (lo > odds) {
                odds = lo;
                y = -3.5f;
            }
            if (hi > odds) {
                odds = hi;
                y = 3.5f;
            }
            odds = lm::lm_powf(odds, 0.5f);
            if (odds + rnd(0.0f, 0.5f) > 0.5f) {
                PlayerCommand c;
                default_command(c);
                c.desiredFunctionType = kFtShot;
                c.useDesiredMovement = false;
                c.useDesiredLookAt = false;
                c.desiredVelocityFloat = rawVel;
                const float shot = stat(kStTechnicalShot);
                float ry = y + rnd(-1.0f + shot, 1.0f - shot);
                c.touchInfo.desiredDirection =
                    (Vec3((kPitchHalfL + 1.0f) * -side, ry, 0) - (pos() + mov() * 0.2f)).normalized(Vec3(-side, 0, 0));
                c.touchInfo.desiredDirection =
                    (c.touchInfo.desiredDirection * 0.7f + -dir() * (float_velocity() / kSprintVel) * 0.3f).normalized();
                c.touchInfo.autoDirectionBias = 1.0f;
                c.touchInfo.desiredPower = rnd(0.7f * (0.6f + goalD * 0.4f), 1.0f * (0.6f + goalD * 0.4f));
                push(c);
            }
        }
        best_dribble_movement(rawDir, rawVel);
    }

    CB_HDNI void add_celebration() {
        int xSide = (ball(0).flat().c[0] > 0) ? 1 : -1;
        int ySide = side;
        const int ltp = team().lastTouchPlayer;
        if (ltp >= 0) ySide = (pos(ltp).c[1] > 0) ? 1 : -1;
        Vec3 cp = Vec3(kPitchHalfL * xSide, kPitchHalfW * ySide, 0);
        Vec3 dd = (cp - pos()).normalized();
        float dv = clamp_velocity((cp - pos()).length() / 4.0f);
        Vec3 dl = pos() + dir() * 1000;
        int ct = 1;
        if (m.lastGoalTeam != team_slot(w, teamID)) {
            ct = 2;
            dv = kIdleVel;
        }
        int made = 1;
        if (ct == 1) {
            if (ltp == player) {
                made = 2;
                dv = kSprintVel;
            } else if (ltp >= 0) {
                if ((pos(ltp) - pos()).length() < 20) {
                    cp = pos(ltp);
                    dd = ((pos(ltp) * 0.5f + cp * 0.5f) - pos()).normalized();
                    dv = clamp_velocity((float)((double)(pos(ltp) - pos()).length() / 2.0));
                } else {
                    dv = kIdleVel;
                }
                dl = pos() + dir(ltp) * 100;
            }
        }
        const uint64_t stop = m.referee.buffer.stopTime;
        if (m.actualTime_ms - stop > 2000 && m.actualTime_ms - stop < 4000) {
            PlayerCommand c;
            default_command(c);
            c.desiredFunctionType = kFtSpecial;
            c.useSpecialVar1 = true;
            c.specialVar1 = ct;
            c.useSpecialVar2 = true;
            c.specialVar2 = made;
            c.useDesiredMovement = false;
            c.useDesiredLookAt = false;
            push(c);
        }
        PlayerCommand c;
        default_command(c);
        c.desiredFunctionType = kFtMovement;
        c.useDesiredMovement = true;
        c.desiredDirection = dd;
        c.desiredVelocityFloat = dv;
        c.useDesiredLookAt = true;
        c.desiredLookAt = dl;
        push(c);
    }

    CB_HDNI void set_piece_commands() {
        const int spt = team_ai().setPieceType;
        PlayerCommand ac;
        default_command(ac);
        if (spt == kGmPenalty) {
            ac.desiredFunctionType = kFtShot;
            ac.useDesiredMovement = false;
            ac.useDesiredLookAt = false;
            float ry = rnd(-5, 5);
            ac.touchInfo.desiredDirection = (Vec3(-side * kPitchHalfL, ry, 0) - pos()).normalized(Vec3(-side, 0, 0));
            ac.touchInfo.desiredPower = rnd(0.4f, 1.0f);
            push(ac);
        } else {
            ac.desiredFunctionType = kFtShortPass;
            ac.useDesiredMovement = false;
            ac.useDesiredLookAt = false;
            ac.touchInfo.inputDirection = dir();
            ac.touchInfo.inputPower = 0.5f;
            ac.touchInfo.autoDirectionBias = 1.0f;
            ac.touchInfo.autoPowerBias = 1.0f;
            ac.touchInfo.forcedTargetPlayer = -1;
            Vec3 dtp;
            bool doCmd = true;
            if (spt == kGmGoalKick) {
                if (rnd(0.0f, 1.0f) > 0.4f && gamer_count_enabled(team()) == 0) {
                    ac.desiredFunctionType = kFtHighPass;
                    float ry = rnd(-kPitchHalfW, kPitchHalfW);
                    dtp = Vec3((kPitchHalfL * -side) * 0.2f, ry, 0.0f);
                } else {
                    ac.desiredFunctionType = kFtShortPass;
                    float ry = rnd(-kPitchHalfW, kPitchHalfW);
                    dtp = Vec3(pos().c[0] * 0.9f, ry, 0.0f);
                }
            } else if (spt == kGmKickOff) {
                ac.desiredFunctionType = kFtShortPass;
                dtp = pos() + dir() * 1.0f;
            } else if (spt == kGmFreeKick) {
                if (rnd(0.0f, 1.0f) > 0.5f) {
                    ac.desiredFunctionType = kFtHighPass;
                    float ry = rnd(-10.0f, 10.0f);
                    dtp = Vec3(kPitchHalfL * -side, ry, 0.0f);
                } else {
                    ac.desiredFunctionType = kFtShortPass;
                    float ry = rnd(-10.0f, 10.0f);
                    dtp = pos() + Vec3(-side * 10.0f, ry, 0.0f);
                }
            } else if (spt == kGmCorner) {
                if (rnd(0.0f, 1.0f) > 0.3f) {
                    ac.desiredFunctionType = kFtHighPass;
                    // GRF evaluates the arguments right to left: y draws first.
                    float ry = rnd(-10.0f, 10.0f);
                    float rx = rnd(0.0f, 0.12f);
                    dtp = Vec3((kPitchHalfL * -side) * (0.99f - rx), ry, 0.0f);
                } else {
                    ac.desiredFunctionType = kFtShortPass;
                    dtp = Vec3((kPitchHalfL * -side) * 0.8f, pos().c[1] * 0.8f, 0.0f);
                }
            } else if (spt == kGmThrowIn) {
                ac.desiredFunctionType = kFtShortPass;
                dtp = pos();
            } else if (m.ballRetainer == player) {
                ac.desiredFunctionType = kFtHighPass;
                float ry = rnd(-kPitchHalfW, kPitchHalfW);
                dtp = Vec3(kPitchHalfL * side, ry, 0.0f);
                int tp = closest_player(s, teamID, dtp, false, player);
                if (tp >= 0) {
                    int co = closest_player(s, oppID, pos(tp), false, -1);
                    if (co >= 0) {
                        if (((pos(co) + mov(co) * 0.1f) - pos(tp)).length() > 10.0f || pl.possessionDuration_ms > 4000)
                            ac.touchInfo.forcedTargetPlayer = tp;
                        else
                            doCmd = false;
                    }
                }
            }
            if (doCmd) {
                TouchInfo &t = ac.touchInfo;
                if (t.forcedTargetPlayer < 0) t.forcedTargetPlayer = closest_player(s, teamID, dtp, false, player);
                get_pass(w, player, ac.desiredFunctionType, t.inputDirection, t.inputPower, t.autoDirectionBias,
                         t.autoPowerBias, t.desiredDirection, t.desiredPower, t.targetPlayer, t.forcedTargetPlayer);
                push(ac);
            }
        }
        if (m.ballRetainer != player) {
            PlayerCommand c;
            default_command(c);
            c.desiredFunctionType = kFtMovement;
            c.useDesiredMovement = true;
            c.useDesiredLookAt = true;
            ball_control_movement(kWalkVel, c.desiredDirection, c.desiredVelocityFloat, c.desiredLookAt);
            push(c);
        } else {
            PlayerCommand c;
            default_command(c);
            c.desiredFunctionType = kFtMovement;
            c.useDesiredMovement = true;
            c.desiredDirection = (ac.touchInfo.desiredDirection.length() > 0.0f)
                                     ? ac.touchInfo.desiredDirection.flat().normalized(dir())
                                     : (Vec3(0) - pos()).normalized(dir());
            c.desiredVelocityFloat = kIdleVel;
            c.useDesiredLookAt = true;
            c.desiredLookAt = pos() + c.desiredDirection * 10.0f;
            push(c);
        }
    }

    CB_HDNI bool request_command() {
        if (m.designatedPossessionPlayer < 0) return s.fail(kStatusUnsupported);
        if (team().designatedTeamPossessionPlayer < 0 || opp_team().designatedTeamPossessionPlayer < 0)
            return s.fail(kStatusUnsupported);
        mi = mental_index(w, ctl.mentalImageTime);
        ctl.lastSwitchTimeDuration_ms = 0;
        ctl.lastSwitchTime_ms = 0;
        pl.desiredTimeToBall_ms = 0;
        controller_situation(w, player, ctl);
        ctl.opponentPlayer = team_best_possession_player(w, oppID);
        ctl.timeNeeded_ms = (float)pl.timeNeededToGetToBall_ms;
        Vec3 rawDir = dir();
        float rawVel = kIdleVel;
        Vec3 manDir = dir();
        float manVel = kIdleVel;
        bool manual = false, extraHaste = false;
        // Laziness is fixed at creation from the player's own entry (GRF).
        const bool lazy = s.ctx.staticData->formation[player].lazy;
        const int role = static_role(player);
        const RefereeBuffer &rb = m.referee.buffer;
        if (!m.inPlay && m.goalScored) {
            add_celebration();
            return true;
        } else if (!m.inPlay && rb.active && (m.referee.foul.foulType == 2 || m.referee.foul.foulType == 3) &&
                   rb.stopTime < m.actualTime_ms - 1000 && rb.prepareTime > m.actualTime_ms) {
            PlayerCommand c;
            default_command(c);
            c.desiredFunctionType = kFtMovement;
            c.useDesiredMovement = true;
            c.useDesiredLookAt = true;
            c.desiredDirection = dir();
            c.desiredVelocityFloat = kIdleVel;
            c.desiredLookAt = m.officials[0].humanoid.spatial.position;
            push(c);
            return true;
        } else if (!m.inPlay || lazy) {
            PlayerCommand c;
            default_command(c);
            c.desiredFunctionType = kFtMovement;
            c.useDesiredMovement = true;
            c.desiredDirection = (dir() * 0.6f + (Vec3(0) - pos()).normalized(dir()) * 0.4f).normalized(dir());
            c.desiredVelocityFloat = clamp_velocity(float_velocity() * 0.95f - rnd(0.0f, 3.2f));
            c.useDesiredLookAt = true;
            c.desiredLookAt = pos() + (ball(0).flat() - pos()).normalized(c.desiredDirection) * 10.0f;
            push(c);
            return true;
        } else if ((m.inSetPiece && team_ai().taker == player) || m.ballRetainer == player) {
            set_piece_commands();
            return true;
        } else if (m.inPlay && !m.inSetPiece && m.ballRetainer != player && m.designatedPossessionPlayer != player &&
                   role != kRoleGK) {
            if (role == kRoleLB || role == kRoleCB || role == kRoleRB)
                field_strategy_input(kDefense, rawDir, rawVel);
            else if (role == kRoleDM || role == kRoleLM || role == kRoleCM || role == kRoleRM || role == kRoleAM)
                field_strategy_input(kMidfield, rawDir, rawVel);
            else if (role == kRoleCF)
                field_strategy_input(kOffense, rawDir, rawVel);
        } else if (m.inPlay && !m.inSetPiece && m.designatedPossessionPlayer == player &&
                   (gamer_count_enabled(team()) == 0 || (!external_active(w, player) && pl.base.externalController >= 0)) &&
                   role != kRoleGK) {
            if (pl.timeNeededToGetToBall_ms < 1000) on_the_ball_commands(rawDir, rawVel);
            extraHaste = false;
        } else if (m.inPlay && !m.inSetPiece && role == kRoleGK) {
            ball_bound_for_goal();
            bool bfg = eliza->ballBoundForGoal;
            if (bfg) manual = true;
            if (player != m.designatedPossessionPlayer) manual = true;
            goalie_input(manDir, manVel);
            if (!ctl.hasUniquePossession || ctl.possessionAmount < 3.4f) {
                bool onlyPickup = false;
                if (!bfg && ctl.possessionAmount > 1.3f) onlyPickup = true;
                keeper_deflect_command(onlyPickup);
            }
            if (pl.timeNeededToGetToBall_ms < 1000 && m.designatedPossessionPlayer == player)
                on_the_ball_commands(rawDir, rawVel);
        }
        bool forceMagnet = false;
        if (m.inPlay && !m.inSetPiece &&
            (team_ai().endApplyTeamPressure_ms > m.actualTime_ms && team_ai().teamPressurePlayer == player) &&
            !ctl.teamHasBestPossession && m.designatedPossessionPlayer != player && role != kRoleGK)
            forceMagnet = true;
        ctl.inputDirection = rawDir;
        ctl.inputVelocityFloat = rawVel;
        eliza->lastDesiredDirection = rawDir.length() != 0 ? rawDir : dir();
        eliza->lastDesiredVelocity = rawVel;
        if (m.inPlay && !m.inSetPiece) {
            ball_control_command();
            trap_command();
            interfere_command(false);
            sliding_command();
        }
        if (!manual && m.inPlay && !m.inSetPiece) {
            const int o = opp_team().designatedTeamPossessionPlayer;
            if (player != m.designatedPossessionPlayer) {
                float ms = mind_set(dynamic_role());
                float hunt = 10.0f + (1.0f - ms) * 10.0f;
                hunt *= 0.5f * pl.base.fatigueFactorInverse +
                        0.5f * (1.0f - nclamp(player_average_velocity(w, player, 10), kIdleVel, kSprintVel));
                hunt *= 0.3f + team_difficulty(w, teamID) * 0.7f;
                if (forceMagnet) {
                    ctl.inputDirection = Vec3(side * kPitchHalfL, 0, 0) - pos();
                    ctl.inputVelocityFloat = kIdleVel;
                    ctl.inputDirection.normalize(dir());
                } else if (!ctl.teamHasBestPossession && pl.manMarking < 0 &&
                           ((pos(o) + mov(o) * 0.12f) - (pos() + mov() * 0.04f)).length() < hunt) {
                    if (player == team().designatedTeamPossessionPlayer && ctl.possessionAmount > 0.8f) {
                        forceMagnet = true;
                        extraHaste = true;
                    }
                    int huntCount = 2;
                    PlayerList cp;
                    closest_players(cp, s, teamID, pos(o) + mov(o) * 0.1f, false, huntCount);
                    bool close = false;
                    for (int i = 0; i < cp.count; i++)
                        if (cp[i] == player) {
                            close = true;
                            break;
                        }
                    if (close) {
                        Vec3 dp = defend_position(o);
                        if (need_defending_movement(side, pos(), dp)) {
                            ctl.inputDirection = (dp - pos()).normalized(ctl.inputDirection);
                            ctl.inputVelocityFloat = clampf_((dp - pos()).length() * kDistToVel, 0.0f, kSprintVel);
                            forceMagnet = true;
                        }
                    }
                }
            }
            ctl.inputVelocityFloat = range_velocity(ctl.inputVelocityFloat);
            movement_command(forceMagnet, extraHaste);
        } else {
            PlayerCommand c;
            default_command(c);
            c.desiredFunctionType = kFtMovement;
            c.useDesiredMovement = true;
            c.desiredDirection = manDir;
            c.desiredVelocityFloat = manVel;
            c.useDesiredLookAt = true;
            c.desiredLookAt = pos() + (mball(40).flat() - pos()).normalized(Vec3(0)) * 10.0f;
            push(c);
        }
        return true;
    }
};

CB_HD void team_apply_team_pressure(const Sim &s, int teamID) {
    Match &w = s.w;
    TeamAIState &ai = team_by_id(w, teamID).ai;
    ai.endApplyTeamPressure_ms = w.m.actualTime_ms + 500;
    int o = team_best_possession_player(w, 1 - teamID);
    const SpatialState &os = hum(w, o).spatial;
    Vec3 op = os.position + os.movement * 0.24f;
    ai.teamPressurePlayer =
        closest_player(s, teamID, op + Vec3(team_side(w, teamID) * 1.0f, 0, 0), true, team_goalie(s, teamID));
    if (ai.teamPressurePlayer >= 0) w.m.players[ai.teamPressurePlayer].manMarking = o;
}
CB_HD void team_apply_keeper_rush(Match &w, int teamID) {
    team_by_id(w, teamID).ai.endApplyKeeperRush_ms = w.m.actualTime_ms + 300;
}

/// Human (external) controller command, ai_controller.h:2250 (HumanRequestCommand).
CB_HDNI bool human_request_command(const Sim &s, int player, CommandQueue &q) {
    Match &w = s.w;
    HumanControllerState &hc = gamer_of(w, player).controller;
    ControllerState &ctl = hc.base;
    AIController e(s, player, q, ctl, nullptr);
    MatchState &m = w.m;
    Player &pl = m.players[player];
    const int teamID = w.playerTeamID[player];
    const TeamAIState &tai = team_by_id(w, teamID).ai;
    const bool *btn = hc.keyboard.buttons;
    auto reset_action = [&]() {
        hc.actionMode = 0;
        hc.gauge_ms = 0;
        hc.actionBufferTime_ms = 0;
    };
    e.mi = mental_index(w, ctl.mentalImageTime);
    pl.desiredTimeToBall_ms = 0;
    ctl.opponentPlayer = team_best_possession_player(w, 1 - teamID);
    ctl.timeNeeded_ms = (float)pl.timeNeededToGetToBall_ms;
    Vec3 rawDir;
    float rawVel = 0;
    keyboard_input(w, player, rawDir, rawVel);
    ctl.inputDirection = rawDir;
    ctl.inputVelocityFloat = rawVel;
    const AnimationState &ca = hum(w, player).anim;
    const int ft = ca.functionType;
    const bool touchPending = ca.frameNumber < ca.touchFrame;
    if (hc.actionMode == 2 && (ft == kFtShortPass || ft == kFtLongPass || ft == kFtHighPass || ft == kFtShot) &&
        !touchPending)
        reset_action();
    if (hc.actionMode == 1 && (ft == kFtSliding || ft == kFtInterfere) && !touchPending) reset_action();
    if (hc.actionMode == 2 && hc.actionButton == kBtnShot && btn[kBtnShortPass] && !m.inSetPiece) reset_action();
    if (hc.actionMode == 2 && hc.actionButton == kBtnHighPass && btn[kBtnShortPass] && !m.inSetPiece) reset_action();
    if (hc.actionMode == 2 && !m.inSetPiece &&
        (hc.actionBufferTime_ms > 2000 ||
         pl.timeNeededToGetToBall_ms > pl.timeNeededToGetToBallPrevious_ms + 700 || ca.functionType == kFtInterfere))
        reset_action();
    if (hc.actionMode == 1 && hc.actionBufferTime_ms > 1000) reset_action();

    if (hc.actionMode == 2) {
        if (!btn[hc.actionButton] || (btn[hc.actionButton] && hc.gauge_ms > 500) ||
            (!pl.hasPossession && !m.inSetPiece && hc.actionBufferTime_ms > 0)) {
            const int baseTime = 60;
            float gauge = (float)(hc.gauge_ms - baseTime) * (1.0f / float(1000 - baseTime));
            gauge = clampf_(gauge, 0.0f, 1.0f);
            auto pass = [&](int passType, float exponent, float autoDir, float autoPow) {
                PlayerCommand c;
                default_command(c);
                c.desiredFunctionType = passType;
                c.useDesiredMovement = false;
                c.useDesiredLookAt = false;
                float ip = clampf_(lm::lm_powf(gauge, exponent), 0.01f, 1.0f);
                TouchInfo &t = c.touchInfo;
                t.inputDirection = ctl.inputDirection;
                t.inputPower = ip;
                t.autoDirectionBias = autoDir;
                t.autoPowerBias = autoPow;
                get_pass(w, player, passType, t.inputDirection, t.inputPower, t.autoDirectionBias, t.autoPowerBias,
                         t.desiredDirection, t.desiredPower, t.targetPlayer, -1);
                queue_push(s, q, c);
            };
            if (m.inSetPiece && tai.taker == player && tai.setPieceType == kGmKickOff) {
                PlayerCommand c;
                default_command(c);
                c.desiredFunctionType = kFtShortPass;
                TouchInfo &t = c.touchInfo;
                t.autoDirectionBias = 1.0f;
                t.autoPowerBias = 1.0f;
                t.inputDirection = e.dir();
                t.inputPower = 0.1f;
                Vec3 tgt = e.pos() + e.dir() * 1.0f;
                t.forcedTargetPlayer = closest_player(s, teamID, tgt, false, player);
                get_pass(w, player, c.desiredFunctionType, t.inputDirection, t.inputPower, t.autoDirectionBias,
                         t.autoPowerBias, t.desiredDirection, t.desiredPower, t.targetPlayer, t.forcedTargetPlayer);
                queue_push(s, q, c);
            } else if (hc.actionButton == kBtnShortPass) {
                pass(kFtShortPass, 0.7f, 0.4f, 0.7f);
            } else if (hc.actionButton == kBtnLongPass) {
                pass(kFtLongPass, 0.65f, 0.2f, 0.7f);
            } else if (hc.actionButton == kBtnHighPass) {
                pass(kFtHighPass, 0.55f, 0.2f, 0.5f);
            } else if (hc.actionButton == kBtnShot) {
                PlayerCommand c;
                default_command(c);
                c.desiredFunctionType = kFtShot;
                c.useDesiredMovement = false;
                c.useDesiredLookAt = false;
                c.desiredVelocityFloat = ctl.inputVelocityFloat;
                c.touchInfo.inputDirection = ctl.inputDirection;
                c.touchInfo.autoDirectionBias = 1.0f;
                c.touchInfo.desiredDirection =
                    shot_direction(w, player, c.touchInfo.inputDirection, c.touchInfo.autoDirectionBias);
                c.touchInfo.desiredPower = clampf_(lm::lm_powf(gauge, 0.6f), 0.01f, 1.0f);
                queue_push(s, q, c);
            }
        }
    } else if (hc.actionMode == 1) {
        if (btn[hc.actionButton]) {
            if (hc.actionButton == kBtnSliding) {
                PlayerCommand c;
                default_command(c);
                c.desiredFunctionType = kFtSliding;
                c.useDesiredMovement = true;
                c.desiredDirection = ctl.inputDirection;
                c.desiredVelocityFloat = ctl.inputVelocityFloat;
                c.useDesiredLookAt = true;
                c.desiredLookAt = e.pos() + e.mov() * 0.1f + c.desiredDirection * 10.0f;
                queue_push(s, q, c);
            }
            if (hc.actionButton == kBtnTeamPressure) team_apply_team_pressure(s, teamID);
            if (hc.actionButton == kBtnKeeperRush) team_apply_keeper_rush(w, teamID);
        } else {
            hc.actionMode = 0;
        }
    }

    if ((m.inSetPiece && tai.taker == player &&
         (hc.actionMode != 2 || (hc.actionMode == 2 && btn[hc.actionButton]) || m.ballRetainer == player)) ||
        (m.inSetPiece && tai.taker != player && m.ballRetainer < 0)) {
        e.set_piece_command();
        return true;
    }

    Vec3 savedNonsteady = ctl.inputDirection;
    ctl.inputDirection = hc.steadyDirection;
    if (m.inPlay && !m.inSetPiece) {
        bool idleTurn = false, knockOn = false;
        if (btn[kBtnDribble]) idleTurn = true;
        if (btn[kBtnDribble] && btn[kBtnSprint]) knockOn = true;
        Vec3 savedDir = ctl.inputDirection;
        float savedVel = ctl.inputVelocityFloat;
        if (hc.actionMode == 2) {
            float dot = e.dir().dot(ctl.inputDirection) * 0.5f + 0.5f;
            if (dot < 0) dot = 0;
            if (e.SPo(player).velocityCategory != kVelIdle)
                ctl.inputDirection = (e.dir() * 1.0f + ctl.inputDirection * 0.0f).normalized(ctl.inputDirection);
            dot = lm::lm_powf(dot, 1.5f);
            dot = dot * 0.8f + 0.2f;
            dot *= 0.9f;
            ctl.inputVelocityFloat = e.float_velocity() * dot;
        }
        e.ball_control_command(idleTurn, knockOn, true, false);
        e.trap_command(idleTurn, knockOn);
        if (hc.actionMode == 2) {
            ctl.inputDirection = savedDir;
            ctl.inputVelocityFloat = savedVel;
        }
        bool byAnyMeans = false;
        if (btn[kBtnPressure]) byAnyMeans = true;
        e.interfere_command(byAnyMeans);
    }
    bool forceMagnet = false, extraHaste = false;
    if (hc.actionMode != 2 && btn[kBtnPressure]) {
        forceMagnet = true;
        extraHaste = true;
    }
    if (hc.actionMode == 2) {
        forceMagnet = true;
        extraHaste = true;
    }
    e.movement_command(forceMagnet, extraHaste);
    if (q.count > 0) {
        PlayerCommand &c = q.el[q.count - 1];
        if (!w.scenario.useMagnet) {
            c.desiredDirection = ctl.inputDirection;
            c.desiredVelocityFloat = ctl.inputVelocityFloat;
            if (c.desiredVelocityFloat < kIdleDribbleSwitch)
                c.desiredDirection = (e.mball(500).flat() - e.pos()).normalized(ctl.inputDirection);
            c.desiredLookAt = e.mball(500).flat();
        }
        if (m.inPlay && !m.inSetPiece && btn[kBtnDribble] && btn[kBtnSprint]) {
            if (!ctl.hasBestPossession) {
                c.desiredDirection = ctl.inputDirection;
                c.desiredVelocityFloat = ctl.inputVelocityFloat;
            }
        }
    }
    ctl.inputDirection = savedNonsteady;
    return true;
}

/// ai_controller.h:2470 (PlayerRequestCommand / ElizaRequestCommand).
CB_HDNI bool player_request_command(const Sim &s, int player, CommandQueue &q) {
    if (external_active(s.w, player)) return human_request_command(s, player, q);
    AIControllerState &st = s.w.m.players[player].base.controller;
    AIController e(s, player, q, st.base, &st);
    return e.request_command();
}

// @@CONTINUE@@

}  // namespace cb
