// cuju-b200: ball-body contacts and player-player bounces, trips and tackles. The pairs are
// processed in GRF's order since each bounce moves players that later pairs read.
//   cuju include/cuju/simulation/collisions.h:23-605
#pragma once

#include "officials.cuh"

namespace cb {

CB_HD float match_last_touch_bias(const Match &w, int decay_ms) {
    int team = w.m.lastTouchTeamID != -1 ? w.m.lastTouchTeamID : w.firstTeamID();
    return team_last_touch_bias(w, team, decay_ms);
}

CB_HDNI bool check_ball_collisions(const Sim &s) {
    Match &w = s.w;
    MatchState &m = w.m;
    if (m.actualTime_ms <= (uint64_t)(uint32_t)(m.lastBodyBallCollisionTime_ms + 150)) return true;
    PlayerList players;
    active_players(players, w, w.firstTeamID());
    {
        PlayerList second;
        active_players(second, w, 1 - w.firstTeamID());
        for (int i = 0; i < second.count; i++) players.push(second[i]);
    }
    Vec3 bounce;
    float bias = 0.0;
    int bounces = 0;
    for (int pi = 0; pi < players.count; pi++) {
        const int p = players[pi];
        const int teamID = w.playerTeamID[p];
        const int thr = 200;
        float oltb = team_last_touch_bias(w, 1 - teamID, thr);
        float ltb = last_touch_bias(w, p, thr);
        if (!(ltb <= 0.01f && oltb > 0.01f)) continue;
        Player &pl = m.players[p];
        const Humanoid &h = pl.base.humanoid;
        const int ft = h.anim.functionType;
        bool collAnim = ft == kFtMovement || ft == kFtTrip || ft == kFtSliding || ft == kFtInterfere || ft == kFtDeflect;
        bool onlyUnexpected = ft == kFtInterfere || ft == kFtDeflect;
        bool unexpected = false;
        if (onlyUnexpected) {
            int ii = mental_index(w, reaction_time_ms(s, p) + h.anim.frameNumber * 10);
            float ud = (mental_ball(w, ii, 1000) - ball_predict(m.ball, 1000)).length();
            if (ud > 0.5f) unexpected = true;
        }
        if (!(collAnim && !pl.hasUniquePossession && onlyUnexpected == unexpected)) continue;
        float bbOff = -0.1f;
        if (!pl.hasPossession) bbOff += 0.03f;
        else bbOff -= 0.03f;
        if (ft == kFtSliding || ft == kFtInterfere) bbOff += 0.1f;
        if (ft == kFtDeflect) bbOff += 0.2f;
        if (!(((h.spatial.position + Vec3(0, 0, 0.8f)) - ball_predict(m.ball, 0)).length() < 2.5f)) continue;
        const Skeleton &sk = s.ctx.skeletons[p];
        Xform xf[kNodes];
        derive_nodes(sk, h.nodes, xf);
        for (int n = 0; n < sk.nodeCount; n++) {
            for (int g = 0; g < sk.nodes[n].geometryCount; g++) {
                WorldGeom wg = geometry_world(sk.nodes[n].geometries[g], xf[n]);
                float br = 0.11f + bbOff;
                if (!wg.box.intersects(ball_predict(m.ball, 0), br)) continue;
                if (p == team_by_id(w, teamID).designatedTeamPossessionPlayer && match_last_touch_bias(w, 200) < 0.01f) {
                    pl.triggerControlledBallCollision = true;
                } else {
                    float mb = oltb * 0.8f + 0.2f;
                    bounce += (ball_predict(m.ball, 0) - wg.position).normalized(Vec3(0)) * mb +
                              h.spatial.movement * (1.0f - mb);
                    bounces++;
                    if (!team_set_last_touch(s, p, kTouchAccidental)) return false;
                    Vec3 bc = wg.box.center();
                    bias += (1.0f - clampf_(((ball_predict(m.ball, 0) - bc).length() - br) / wg.box.radius(), 0.0f, 1.0f)) *
                                0.9f +
                            0.1f;
                }
            }
        }
    }
    if (bias > 0.0f) {
        bounce /= Vec3(bounces * 1.0f);
        bounce.c[2] *= 0.6f;
        bounce.normalize();
        Vec3 cur = m.ball.momentum;
        Vec3 full = (bounce * 6.0f) + (bounce * cur.length() * 0.6f) + (cur * -0.2f);
        bias = clampf_(bias, 0.0f, 1.0f);
        bias = bias * 0.5f + 0.5f;
        Vec3 res = full * bias + cur * (1.0f - bias);
        if (res.length() > cur.length()) res = res.normalized(Vec3(0)) * cur.length();
        res *= 0.7f;
        ball_touch(s, res);
        // GRF evaluates the arguments right to left: z, then y, then x.
        float rz = random_in_range(w.rng, -30, 30);
        float ry = random_in_range(w.rng, -30, 30);
        float rx = random_in_range(w.rng, -30, 30);
        ball_set_rotation(w, rx, ry, rz, 0.5f * bias);
        m.lastBodyBallCollisionTime_ms = (uint32_t)m.actualTime_ms;
    }
    return true;
}

// The position in the fixed pitch frame, in which team 0 starts on side -1.
CB_HD Vec3 pitch_position(const Match &w, int p) {
    Vec3 pos = hum(w, p).spatial.position;
    const int teamID = w.playerTeamID[p];
    const int side = w.flags.teamSide[teamID];
    bool original = teamID == 0 ? (side == -1) : (side == 1);
    if (!original) pos.mirror();
    return pos;
}

CB_HDNI void referee_trip_notice(Match &w, int tripped, int tripping, int tackleType) {
    MatchState &m = w.m;
    Referee &ref = m.referee;
    if (ref.buffer.active) return;
    const Humanoid &th = hum(w, tripped), &gh = hum(w, tripping);
    const int tt = w.playerTeamID[tripped], gt = w.playerTeamID[tripping];
    if (tackleType == 2) {
        if ((double)team_by_id(w, tt).fadingTeamPossessionAmount > 1.1 &&
            (gh.anim.functionType == kFtInterfere || gh.anim.functionType == kFtSliding) &&
            (double)(th.spatial.position - ball_predict(m.ball, 0).flat()).length() < 2.0 && gt != tt) {
            ref.foul.foulType = 1;
            ref.foul.advantage = true;
            ref.foul.foulPlayer = tripping;
            ref.foul.foulVictim = tripped;
            ref.foul.foulTime = m.actualTime_ms;
            ref.foul.foulPosition = pitch_position(w, tripped);
            ref.foul.hasBeenProcessed = false;
        }
    } else if (tackleType == 3 && (tripping != ref.foul.foulPlayer || ref.foul.foulType == 0)) {
        if (m.actualTime_ms - m.players[tripping].base.lastTouchTime_ms > 600 && gh.anim.functionType == kFtSliding &&
            gt != tt && (double)(ball_predict(m.ball, 0) - th.spatial.position).length() < 8.0) {
            float severity = 1.0;
            if (gh.anim.touchFrame != -1) {
                const int tf = gh.anim.touchFrame, cf = gh.anim.frameNumber;
                float timing = clampf_((float)(fabs((double)(tf - cf)) / tf), 0.0, 1.0);
                severity = (float)(lm::lm_pow((double)timing, 0.7) * 0.5);
                severity = (float)(severity + nclamp((ball_predict(m.ball, 0) - gh.anim.touchPosition).length(), 0.0, 2.0) * 0.5);
            }
            // GRF adds `dot * 0.5 + 0.5` to the severity as one double term.
            severity = (float)(severity +
                               ((th.spatial.position - gh.spatial.position).normalized(Vec3(0)).dot(th.spatial.directionVector) *
                                    0.5 +
                                0.5));
            if ((double)severity > 1.0) {
                ref.foul.foulType = 1;
                ref.foul.advantage = false;
                ref.foul.foulPlayer = tripping;
                ref.foul.foulVictim = tripped;
                ref.foul.foulTime = m.actualTime_ms;
                ref.foul.foulPosition = pitch_position(w, tripped);
                ref.foul.hasBeenProcessed = false;
                if ((double)severity > 1.4) ref.foul.foulType = 2;
                if ((double)severity > 2.0) ref.foul.foulType = 3;
            }
        }
    }
}

CB_HDNI void trip_me(const Sim &s, int p, const Vec3 &trip, int tripType) {
    Match &w = s.w;
    if (w.m.ballRetainer == p) return;
    Humanoid &h = w.m.players[p].base.humanoid;
    const Anim &pa = s.A(h.anim.anim);
    if (pa.incomingSpecialState != kSS_Empty || pa.outgoingSpecialState != kSS_Empty) return;
    if (h.interruptAnim == kIntNone &&
        (h.anim.functionType != kFtTrip || (s.D(h.anim.anim).tripTypeIsOne && tripType > 1)) &&
        h.anim.functionType != kFtSliding) {
        h.interruptAnim = kIntTrip;
        h.tripDirection = trip;
        h.tripType = tripType;
    }
}

struct Bounce {
    int opponent;
    float force;
};
using BounceList = List<Bounce, kPlayers>;

CB_HD bool boxes_intersect(const Aabb &b, const Aabb &o) {
    return (o.mn.c[0] < b.mx.c[0] && o.mn.c[1] < b.mx.c[1] && o.mn.c[2] < b.mx.c[2]) &&
           (o.mx.c[0] > b.mn.c[0] && o.mx.c[1] > b.mn.c[1] && o.mx.c[2] > b.mn.c[2]);
}
struct PlayerGeom {
    bool footOrLowerLeg;
    WorldGeom wg;
};
using PlayerGeomList = List<PlayerGeom, kNodes * 2>;
CB_HDNI void player_geometries(const Sim &s, int p, PlayerGeomList &out) {
    const Skeleton &sk = s.ctx.skeletons[p];
    Xform xf[kNodes];
    derive_nodes(sk, hum(s.w, p).nodes, xf);
    out.count = 0;
    for (int n = 0; n < sk.nodeCount; n++)
        for (int g = 0; g < sk.nodes[n].geometryCount; g++)
            out.push(PlayerGeom{sk.nodes[n].geometries[g].footOrLowerLeg, geometry_world(sk.nodes[n].geometries[g], xf[n])});
}

CB_HDNI void check_humanoid_collision(const Sim &s, int a, int b, BounceList &ab, BounceList &bb) {
    Match &w = s.w;
    MatchState &m = w.m;
    const float distF = 0.72f;
    const float bounceR = 0.5f * distF;
    const float similarR = 0.8f * distF;
    const float similarExp = 0.2f;
    const float similarForceF = 0.25f;
    auto SP = [&](int p) -> const SpatialState & { return hum(w, p).spatial; };
    auto st = [&](int p, int k) { return statistic(s, p, k); };
    auto ftOf = [&](int p) { return hum(w, p).anim.functionType; };
    auto pending = [&](int p) { return hum(w, p).anim.frameNumber < hum(w, p).anim.touchFrame; };
    auto designated = [&](int p) { return team_by_id(w, w.playerTeamID[p]).designatedTeamPossessionPlayer; };
    Vec3 pa = SP(a).position, pb = SP(b).position;
    float dist = (pa - pb).length();
    float bb_bias = 0.0f;
    Vec3 bv;
    float aBack = 0.5f, bBack = 0.5f;
    if (dist < bounceR * 2.0f || dist < (bounceR + similarR) * 2.0f) {
        bv = (pa - pb).normalized(Vec3(0, -1, 0));
        Vec3 af = rot2d(SP(a).directionVector, SP(a).relBodyAngle.value() * 0.7f);
        Vec3 bf = rot2d(SP(b).directionVector, SP(b).relBodyAngle.value() * 0.7f);
        aBack = clampf_(af.dot(bv) * 0.5f + 0.5f, 0.0f, 1.0f);
        bBack = clampf_(bf.dot(-bv) * 0.5f + 0.5f, 0.0f, 1.0f);
        auto ballDistDiff = [&]() {
            float ad = (ball_predict(m.ball, 10).flat() - SP(a).position).length();
            float bd = (ball_predict(m.ball, 10).flat() - SP(b).position).length();
            float bc = std_min(bd, 1.2f), ac = std_min(ad, 1.2f);
            return clampf_(bc - ac, -0.6f, 0.6f) * 1.0f;
        };
        if (dist < bounceR * 2.0f) {
            bb_bias += aBack * 0.8f;
            bb_bias -= bBack * 0.8f;
            float av = player_float_velocity(w, a), bvv = player_float_velocity(w, b);
            bb_bias -= clampf_(((av - bvv) / kSprintVel) * 0.2f, -0.2f, 0.2f);
            if (pending(a) && ftOf(a) == kFtInterfere) bb_bias += 0.1f + 0.4f * st(a, kStTechnicalStandingTackle);
            if (pending(a) && ftOf(a) == kFtSliding) bb_bias += 0.1f + 0.4f * st(a, kStTechnicalSlidingTackle);
            if (pending(b) && ftOf(b) == kFtInterfere) bb_bias -= 0.1f + 0.4f * st(b, kStTechnicalStandingTackle);
            if (pending(b) && ftOf(b) == kFtSliding) bb_bias -= 0.1f + 0.4f * st(b, kStTechnicalSlidingTackle);
            if (a == m.designatedPossessionPlayer) bb_bias += 0.4f;
            if (b == m.designatedPossessionPlayer) bb_bias -= 0.4f;
            if (a == designated(a) && b == designated(b)) bb_bias += ballDistDiff();
            bb_bias += st(a, kStPhysicalBalance) * 1.0f;
            bb_bias -= st(b, kStPhysicalBalance) * 1.0f;
            bb_bias = clampf_(bb_bias, -1.0f, 1.0f);
            bb_bias *= 0.5f;
            float nb = bb_bias * 0.5f + 0.5f;
            Vec3 ao = (pa - pb).normalized(Vec3(0)) * (bounceR - dist * 0.5f) * (1.0f - nb) * 2.0f;
            Vec3 bo = (pb - pa).normalized(Vec3(0)) * (bounceR - dist * 0.5f) * nb * 2.0f;
            if (m.designatedPossessionPlayer == b && m.players[b].hasPossession) {
                Vec3 lp = pb + rot2d(SP(b).directionVector, 0.3f * kPi) * bounceR * 2;
                Vec3 rp = pb + rot2d(SP(b).directionVector, -0.3f * kPi) * bounceR * 2;
                Vec3 near = (pa - lp).length() < (pa - rp).length() ? lp : rp;
                ao += normalized_max(near - pa, 0.01f) * st(a, kStPhysicalBalance) * 0.3f;
            } else if (m.designatedPossessionPlayer == a && m.players[a].hasPossession) {
                Vec3 lp = pa + rot2d(SP(a).directionVector, 0.3f * kPi) * bounceR * 2;
                Vec3 rp = pa + rot2d(SP(a).directionVector, -0.3f * kPi) * bounceR * 2;
                Vec3 near = (pb - lp).length() < (pb - rp).length() ? lp : rp;
                bo += normalized_max(near - pb, 0.01f) * st(b, kStPhysicalBalance) * 0.3f;
            }
            normalize_max(ao, kSprintVel * 0.01f);
            normalize_max(bo, kSprintVel * 0.01f);
            offset_position(w, a, ao);
            offset_position(w, b, bo);
        }
        float simBias = 0.0f;
        if (similarForceF > 0.0f && dist < (bounceR + similarR) * 2.0f) {
            float gap = dist - bounceR * 2.0f;
            float shell = (0.0f < gap) ? gap : 0.0f;
            simBias += aBack * 0.8f;
            simBias -= bBack * 0.8f;
            float av = player_float_velocity(w, a), bvv = player_float_velocity(w, b);
            simBias -= clampf_(((av - bvv) / kSprintVel) * 0.2f, -0.2f, 0.2f);
            if (a == m.designatedPossessionPlayer) simBias += 0.6f;
            if (b == m.designatedPossessionPlayer) simBias -= 0.6f;
            if (a == designated(a) && b == designated(b)) simBias += ballDistDiff();
            simBias += st(a, kStPhysicalBalance) * 1.0f;
            simBias -= st(b, kStPhysicalBalance) * 1.0f;
            simBias = clampf_(simBias, -1.0f, 1.0f);
            simBias *= 0.9f;
            float sf = clampf_(1.0f - (shell / (similarR * 2.0f)), 0.0f, 1.0f);
            sf = lm::lm_powf(sf, similarExp);
            sf *= similarForceF;
            float ns = simBias * 0.5f + 0.5f;
            ab.push(Bounce{b, sf * (1.0f - ns)});
            bb.push(Bounce{a, sf * ns});
        }
        if (dist < bounceR * 2.0f) {
            float as = 0.0f, bs = 0.0f;
            as += (1.0f - aBack) * 1.0f;
            bs += (1.0f - bBack) * 1.0f;
            float av = player_float_velocity(w, a), bvv = player_float_velocity(w, b);
            as += nclamp(av, kIdleVel, kSprintVel) * 1.0f;
            bs += nclamp(bvv, kIdleVel, kSprintVel) * 1.0f;
            if (m.players[a].hasBestPossession) as += 1.0f;
            if (m.players[b].hasBestPossession) bs += 1.0f;
            float balW = 3.0f;
            as += (1.0f - st(a, kStPhysicalBalance) * 1.0f) * balW;
            bs += (1.0f - st(b, kStPhysicalBalance) * 1.0f) * balW;
            as += clampf_(hum(w, a).decayingPositionOffset.length() * 10.0f, 0.0f, 1.0f);
            bs += clampf_(hum(w, b).decayingPositionOffset.length() * 10.0f, 0.0f, 1.0f);
            float penW = 6.0f;
            float pen = ((SP(a).position + SP(a).movement * 0.03f) - (SP(b).position + SP(b).movement * 0.03f)).length();
            as += lm::lm_powf(1.0f - nclamp(pen, 0.0f, bounceR * 2.0f), 0.4f) * penW;
            bs += lm::lm_powf(1.0f - nclamp(pen, 0.0f, bounceR * 2.0f), 0.4f) * penW;
            float abd = (ball_predict(m.ball, 10).flat() - SP(a).position).length();
            float bbd = (ball_predict(m.ball, 10).flat() - SP(b).position).length();
            as += 1.0f - nclamp(abd, 0.0f, 0.7f);
            bs += 1.0f - nclamp(bbd, 0.0f, 0.7f);
            as /= 5.0f + balW + penW;
            bs /= 5.0f + balW + penW;
            const float t0 = 0.38f, t1 = 0.48f, t2 = 0.58f;
            if (as > t0) {
                int tt = 0;
                if (as > t1) tt = 1;
                if (as > t2) tt = 2;
                if (tt > 0) {
                    trip_me(s, a, (SP(a).movement * 0.1f + SP(b).movement * 0.06f + bv * 1.0f).normalized(bv), tt);
                    referee_trip_notice(w, a, b, tt);
                }
            }
            if (bs > t0) {
                int tt = 0;
                if (bs > t1) tt = 1;
                if (bs > t2) tt = 2;
                if (tt > 0) {
                    trip_me(s, b, (SP(b).movement * 0.1f + SP(a).movement * 0.06f - bv * 1.0f).normalized(-bv), tt);
                    referee_trip_notice(w, b, a, tt);
                }
            }
        }
    }
    auto frameOf = [&](int p) { return hum(w, p).anim.frameNumber; };
    auto frameCountOf = [&](int p) { return s.A(hum(w, p).anim.anim).frameCount; };
    int tackle = 0;
    if ((ftOf(a) == kFtSliding || ftOf(a) == kFtInterfere) && frameOf(a) > 5 && frameOf(a) < 28) tackle += 1;
    if ((ftOf(b) == kFtSliding || ftOf(b) == kFtInterfere) && frameOf(b) > 5 && frameOf(b) < 28) tackle += 2;
    if (dist < 2.0f && tackle > 0 && tackle < 3) {
        const int tackler = tackle == 1 ? a : b, victim = tackle == 1 ? b : a;
        PlayerGeomList tg, vg;
        player_geometries(s, tackler, tg);
        player_geometries(s, victim, vg);
        for (int i = 0; i < tg.count; i++) {
            Aabb tb = tg[i].wg.box;
            tb.mn += 0.1f;
            tb.mx -= Vec3(0.1f);
            for (int j = 0; j < vg.count; j++) {
                if (vg[j].footOrLowerLeg) {
                    if (boxes_intersect(tb, vg[j].wg.box)) {
                        if (frameOf(tackler) > 10 && frameOf(tackler) < frameCountOf(tackler) - 6) {
                            Vec3 tv = SP(victim).directionVector;
                            int tt = 3;
                            if (ftOf(tackler) == kFtInterfere) tt = 1;
                            trip_me(s, victim, tv, tt);
                            referee_trip_notice(w, victim, tackler, tt);
                        }
                        break;
                    }
                }
            }
        }
    }
}

CB_HDNI bool check_humanoid_collisions(const Sim &s) {
    Match &w = s.w;
    PlayerList players;
    active_players(players, w, w.firstTeamID());
    {
        PlayerList second;
        active_players(second, w, 1 - w.firstTeamID());
        for (int i = 0; i < second.count; i++) players.push(second[i]);
    }
    BounceList bl[kPlayers];
    for (int i = 0; i < players.count; i++) bl[i].count = 0;
    for (int i = 0; i + 1 < players.count; i++)
        for (int j = i + 1; j < players.count; j++) check_humanoid_collision(s, players[i], players[j], bl[i], bl[j]);
    for (int i = 0; i < players.count; i++) {
        float total = 0.0f;
        for (int k = 0; k < bl[i].count; k++) total += bl[i][k].force;
        if (total > 0.0f) {
            Vec3 v;
            for (int k = 0; k < bl[i].count; k++)
                v += (hum(w, bl[i][k].opponent).spatial.movement - hum(w, players[i]).spatial.movement) *
                     bl[i][k].force * (bl[i][k].force / total);
            offset_position(w, players[i], v * 0.01f * 1.0f);
        }
    }
    return true;
}

}  // namespace cb
