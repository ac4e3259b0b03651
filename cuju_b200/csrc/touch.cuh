// cuju-b200: the ball's per-tick process, touches, and the touch vectors of passes, shots and
// ball control (their RNG draws happen in GRF's order).
//   ball process / touch      cuju include/cuju/simulation/ball_touch.h:17-139
//   touch vectors             cuju include/cuju/simulation/touch.h:18-397
#pragma once

#include "rng.cuh"
#include "select.cuh"

namespace cb {

CB_HD void ball_recalc(Match &w) {
    ball_materialize(w.m.ball);
    BallMotion unused;
    ball_predict_path(w.m.ball, w.m.ballIsInGoal, unused);
}

// The outcome of a second ball_recalc right after one that computed every entry (an empty cache,
// as ball_touch makes it) on the same inputs (momentum, position, orientation and spin buffers
// unchanged, no lazy mirror pending), without running the flight again. Its first step lands on
// predictions[1] again (with the same orientation prediction and net touch), so its cache test
// reads predictions[2] == predictions[1]. Where that holds it shifts entries 2..399 down by one,
// as a cached run does; otherwise it recomputes every later step from the same inputs, which gives
// back the entries already there.
CB_HD void ball_recalc_again(Ball &b) {
    if (!(b.validPredictions > 0 && b.predictions[2] == b.predictions[1])) {
        b.validPredictions = (int32_t)kCachedPredictions;
        return;
    }
    b.validPredictions--;
    const int last = (int)(kPredictionSpan_ms + kCachedPredictions * 10) / 10 - 1;  // 399
#if CB_DEVICE_PASS
    if (!crew_serial()) {
        // One block of entries per pass, one entry per lane: each lane reads its source before the
        // barrier and writes one place down after it; a pass writes only below what later passes read.
        const int w = crew_width();
        for (int base = 2; base <= last; base += w) {
            const int e = base + crew_rank();
            Vec3 v;
            if (e <= last) v = b.predictions[e + 1];
            crew_sync();
            if (e <= last) b.predictions[e] = v;
            crew_sync();
        }
        return;
    }
#endif
    for (int e = 2; e <= last; e++) b.predictions[e] = b.predictions[e + 1];
}

// One tick of the ball: predict, advance one step, append the position history (401 entries).
CB_HDNI void ball_process(Ball &b, bool inGoal) {
    ball_materialize(b);
    BallMotion bm;
    ball_predict_path(b, inGoal, bm);
    b.momentum = bm.momentum;
    b.rotationPerMs = bm.rotationPerMs;
    b.positionBuffer = predict_at(b.predictions, 10);
    b.orientationBuffer = b.orientationPrediction;
    auto &hist = b.positionHistory;
    if (hist.count < (int)kBallHistory) {
        hist[hist.count++] = b.positionBuffer;
    } else {
        const int n = hist.count;
#if CB_DEVICE_PASS
        if (!crew_serial()) {
            // A crew moves one block of entries per pass, one entry per lane: every lane reads its
            // entry before the barrier and writes it one place down after it. A pass writes only
            // below the entries later passes read.
            const int w = crew_width();
            for (int base = 1; base < n; base += w) {
                const int e = base + crew_rank();
                Vec3 v;
                if (e < n) v = hist[e];
                crew_sync();
                if (e < n) hist[e - 1] = v;
                crew_sync();
            }
        } else
#endif
        {
            for (int e = 1; e < n; e++) hist[e - 1] = hist[e];
        }
        hist[n - 1] = b.positionBuffer;
    }
}

CB_HDNI void team_possession_stats(const Sim &s, int teamID) {
    Match &w = s.w;
    crew_for(w.m.playerCount, [&](int p) {
        if (w.playerTeamID[p] == teamID && w.m.players[p].base.isActive)
            update_possession_stats(w, *s.ctx.staticData, p);
    });
    Team &t = team_by_id(w, teamID);
    t.hasPossession = false;
    t.timeNeededToGetToBall_ms = 100000;
    for (int p = 0; p < w.m.playerCount; p++) {
        if (w.playerTeamID[p] != teamID || !w.m.players[p].base.isActive) continue;
        const Player &pl = w.m.players[p];
        if (pl.hasPossession) t.hasPossession = true;
        if ((int)pl.timeNeededToGetToBall_ms < t.timeNeededToGetToBall_ms)
            t.timeNeededToGetToBall_ms = (int)pl.timeNeededToGetToBall_ms;
    }
}

// The ball takes `target` as its momentum; predictions run twice (GRF recomputes once for the
// momentum and once for the touch, and the cached-prediction count depends on both).
CB_HDNI void ball_touch(const Sim &s, const Vec3 &target) {
    Match &w = s.w;
    Ball &b = w.m.ball;
    b.validPredictions = 0;
    if (b.positionBuffer.c[2] < 0.11f) b.positionBuffer.c[2] = 0.11f;
    b.momentum = target;
    ball_recalc(w);
    ball_recalc_again(b);
    if (w.m.mentalImages.count > 0) {
        MentalImage &im = w.m.mentalImages[0];
        im.ballPredictions.count = kPredictionSpan_ms / 10;
        for (int i = 0; i < (int)(kPredictionSpan_ms / 10); i++) im.ballPredictions[i] = b.predictions[i];
        im.lazyFlip = b.lazyFlip;
    }
    team_possession_stats(s, w.firstTeamID());
    team_possession_stats(s, 1 - w.firstTeamID());
}

CB_HD void ball_set_rotation(Match &w, float x, float y, float z, float bias = 1.0f) {
    Quat rx, ry, rz;
    rx.set_angle_axis(clampf_(x * 0.001f, -kPi * 0.49f, kPi * 0.49f), Vec3(-1, 0, 0));
    ry.set_angle_axis(clampf_(y * 0.001f, -kPi * 0.49f, kPi * 0.49f), Vec3(0, 1, 0));
    rz.set_angle_axis(clampf_(z * 0.001f, -kPi * 0.49f, kPi * 0.49f), Vec3(0, 0, 1));
    Quat tmp = rx * ry * rz;
    Ball &b = w.m.ball;
    b.rotationPerMs = b.rotationPerMs.slerp(bias, tmp);
    ball_recalc(w);
}
CB_HD void ball_set_position(Match &w, const Vec3 &target) {
    Ball &b = w.m.ball;
    b.validPredictions = 0;
    b.positionBuffer = target;
    b.momentum = Vec3(0);
    ball_set_rotation(w, 0, 0, 0, 1.0f);
    b.positionHistory.count = 0;
}

CB_HDNI bool referee_ball_touched(const Sim &s);  // referee.cuh

CB_HD bool team_set_last_touch(const Sim &s, int p, int touchType) {
    Match &w = s.w;
    const int teamID = w.playerTeamID[p];
    team_by_id(w, teamID).lastTouchPlayer = p;
    Player &pl = w.m.players[p];
    pl.base.lastTouchTime_ms = w.m.actualTime_ms;
    pl.base.lastTouchType = touchType;
    w.m.lastTouchTeamIDs[touchType] = teamID;
    w.m.lastTouchTeamID = teamID;
    return referee_ball_touched(s);
}

// ---------------------------------------------------------------------------------------------
// Touch vectors.
CB_HD float controller_velocity(Match &w, int p) {
    if (external_active(w, p)) return keyboard_velocity(w, p);
    return w.m.players[p].base.controller.lastDesiredVelocity;
}

CB_HDNI void difficulty_factors(const Sim &s, int p, const Vec3 &posOffset, float &df, float &hf, float &bmf) {
    Match &w = s.w;
    const Ball &b = w.m.ball;
    const SpatialState &sp = hum(w, p).spatial;
    df = 0.0f;
    hf = 0.0f;
    bmf = 0.0f;
    float offPen = nclamp(posOffset.length(), 0.0f, 0.1f) * 2.0f;
    float velPen = lm::lm_powf(nclamp((sp.movement - b.momentum).length(), 10.0f, 50.0f), 1.5f) * 5.0f;
    float nd = nclamp(((sp.position + sp.directionVector * 0.2f) - ball_predict(b, 0).flat()).length(), 0.7f, 1.3f);
    float farPen = nd * nd * 2.0f;
    df += offPen * 2.0f;
    df += velPen;
    df += farPen * 4.0f;
    hf += offPen * 0.5f;
    hf += velPen * 2.0f;
    hf += farPen;
    const int teamID = w.playerTeamID[p];
    if (w.m.lastTouchTeamID != teamID) {
        int ltp = team_by_id(w, 1 - teamID).lastTouchPlayer;
        if (ltp >= 0) {
            int decay = cvt_f_i32(1000 - statistic(s, p, kStPhysicalReaction) * 500);
            float pen = lm::lm_powf(last_touch_bias(w, ltp, decay), 0.6f) * 5.0f;
            df += pen;
            hf += pen;
            bmf += pen * 0.1f;
        }
    }
    bmf = clampf_(bmf, 0.0f, 0.9f);
    float skill = (1.0f - statistic(s, p, kStTechnicalBallControl) * 0.5f) * random_in_range(w.rng, 0.5f, 1.0f);
    df *= skill;
    hf *= skill;
    bmf *= skill;
    df = clampf_(df, 0.0f, 1.0f);
    hf = clampf_(hf, 0.0f, 1.0f);
    bmf = clampf_(bmf, 0.0f, 1.0f);
}

CB_HDNI bool ball_control_vector(const Sim &s, int p, const Vec3 &nextStartPos, float nextStartAngle,
                                 float nextBodyAngle, const Vec3 &outMov, const AnimationState &ca,
                                 int frameNumber, const SpatialState &sp, float &xr, float &yr, Vec3 &touch,
                                 float extraFootDist = 0.0f) {
    Match &w = s.w;
    const Ball &b = w.m.ball;
    const Player &pl = w.m.players[p];
    const Anim &a = s.A(ca.anim);
    const PlayerCommand &oc = ca.originatingCommand;
    auto st = [&](int k) { return statistic(s, p, k); };
    float physicsBias = 0.7f;
    if (!pl.hasPossession) physicsBias = 0.9f;
    if (vel_category(a.outgoingVelocity) == kVelIdle) physicsBias = 1.0f;
    float expl = 0.6f;
    float maxOver = 1.0f * expl;
    if (oc.desiredVelocityFloat < kDribbleWalkSwitch) maxOver = 0.0f;
    if (oc.desiredVelocityFloat > kWalkSprintSwitch) maxOver = 2.0f * expl;
    float cdf = sp.directionVector.dot(oc.desiredDirection) * 0.5f + 0.5f;
    float ndf = rot2d(Vec3(0, -1, 0), nextStartAngle).dot(oc.desiredDirection) * 0.5f + 0.5f;
    float dotF = clampf_(std_min(cdf, ndf), 0.0f, 1.0f);
    maxOver *= dotF;
    if (vel_category(a.outgoingVelocity) == kVelIdle) maxOver = 0.0f;
    float origBias = 0.7f;
    float cv = controller_velocity(w, p);
    Vec3 desMov = oc.desiredDirection * (oc.desiredVelocityFloat * origBias + cv * (1.0f - origBias));
    if (desMov.length() > kWalkSprintSwitch)
        desMov = desMov.normalized(Vec3(0)) *
                 stretch_sprint(desMov.length(), kSprintVel, max_velocity(*s.ctx.staticData, p));
    float vel = clampf_(desMov.length(), outMov.length(), outMov.length() + maxOver);
    desMov = desMov.normalized(rot2d(Vec3(0, -1, 0), nextStartAngle)) * vel;
    Vec3 physMov = rot2d(Vec3(0, -1, 0), nextStartAngle) * vel;
    float desVel = desMov.length();
    float physVel = physMov.length();
    Vec3 relFoot = front_of_foot_offset(physVel, nextBodyAngle - sp.angle.value(), ball_predict(b, 0).c[2]);
    float annoyVel = curve(nclamp(a.outgoingVelocity, kIdleVel, kSprintVel), 0.7f);
    float oppAnnoy = (1.0f - nclamp(closest_opponent_distance(s, p), 0.5f, 1.5f)) *
                     (1.0f - (st(kStMentalCalmness) * 0.5f + st(kStPhysicalBalance) * 0.3f)) * annoyVel;
    Vec3 foot = rot2d(Vec3(0, -1, 0), nextBodyAngle) * (relFoot.length() + extraFootDist + oppAnnoy * 3.0f);
    float hff = nclamp(ball_predict(b, 0).c[2], 0.5f, 1.0f) * 0.5f;
    foot += relFoot * hff * 0.5f + sp.bodyDirectionVector * hff * 0.5f;
    Vec3 desBall = nextStartPos, physBall = nextStartPos;
    float dvf = nclamp(desVel, 0.0f, kSprintVel);
    float desDelay = dvf * dvf * 0.60f + 0.25f;
    float pvf = nclamp(physVel, 0.0f, kSprintVel);
    float physDelay = pvf * pvf * 0.60f + 0.25f;
    desBall += desMov * desDelay + foot;
    physBall += physMov * physDelay + foot;
    Vec3 planned = physBall * physicsBias + desBall * (1.0f - physicsBias);
    Vec3 toPlanned = planned - ball_predict(b, 0).flat();
    float ttg = (((a.frameCount - 1) - frameNumber) * 10) * 0.001f;
    ttg += physDelay * physicsBias + desDelay * (1.0f - physicsBias);
    ttg += kTouchOffset_ms * 0.001f;
    float divisor = ttg * (0.38f + 0.02f * st(kStTechnicalDribble));
    divisor *= 1.1f;
    float power = lm::lm_powf((toPlanned.length() / divisor), 0.7f);
    Vec3 dir = toPlanned.normalized(rot2d(Vec3(0, -1, 0), nextBodyAngle));
    float height = clampf_(0.1f + 1.5f * lm::lm_powf(power / 10.0f, 1.6f), 0.0f, 1.5f);
    float pm = 1.2f - (st(kStTechnicalBallControl) * 0.03f);
    float vb = nclamp(vel, kWalkVel, kSprintVel - 0.8f);
    pm = 1.0f * (1.0f - vb) + pm * vb;
    touch = dir * power * pm + Vec3(0, 0, height);
    float backspin = 30.0f;
    float tv = touch.length();
    float vf = lm::lm_powf(nclamp(touch.length(), 0.0f, 10.0f), 0.7f);
    Vec3 spinDir = (foot.normalized(Vec3(0)) * 0.6f + touch.normalized(Vec3(0)) * 0.4f).normalized(Vec3(0));
    xr = spinDir.c[1] * ((2 * kPi * tv) - (backspin * vf));
    yr = spinDir.c[0] * ((2 * kPi * tv) - (backspin * vf));
    return true;
}

CB_HDNI bool trap_vector(const Sim &s, int p, const Vec3 &nextStartPos, float nextStartAngle,
                         float nextBodyAngle, const Vec3 &outMov, const AnimationState &ca, int frameNumber,
                         const SpatialState &sp, const Vec3 &posOffset, float &xr, float &yr, Vec3 &result) {
    float df, hf, bmf;
    difficulty_factors(s, p, posOffset, df, hf, bmf);
    Vec3 bc;
    if (!ball_control_vector(s, p, nextStartPos, nextStartAngle, nextBodyAngle, outMov, ca, frameNumber, sp, xr,
                             yr, bc, df))
        return false;
    const Vec3 bm = s.w.m.ball.momentum;
    bc.c[2] += bm.c[2] * hf * 1.0f + hf * 4.0f;
    result = bc * (1.0f - bmf) + bm * bmf;
    return true;
}

CB_HDNI Vec3 shot_vector(const Sim &s, int p, const AnimationState &ca, const SpatialState &sp,
                         const Vec3 &posOffset, float &xr, float &yr, float &zr) {
    Match &w = s.w;
    const Anim &a = s.A(ca.anim);
    const AnimDerived &d = s.D(ca.anim);
    const PlayerCommand &oc = ca.originatingCommand;
    const Vec3 bm = w.m.ball.momentum;
    auto st = [&](int k) { return statistic(s, p, k); };
    uint8_t *rng = w.rng;
    Vec3 touchMov = rot2d(movement_at_frame(s.T().positions + a.firstPosition, a.positionCount, ca.frameNumber, 0),
                          sp.angle.value());
    Vec3 touchDir = touchMov.normalized(sp.directionVector);
    float touchVel = touchMov.length();
    if (vel_category(touchVel) == kVelIdle) touchDir = sp.directionVector;
    float ideal = 0.2f * kPi;
    float negOff = fabsf(angle2d_to(touchDir, rot2d(oc.touchInfo.desiredDirection, -ideal)));
    float posOff = fabsf(angle2d_to(touchDir, rot2d(oc.touchInfo.desiredDirection, ideal)));
    float angle = (posOff < negOff) ? posOff : negOff;
    float dirF = clampf_(angle / kPi, 0.0f, 1.0f);
    dirF = curve(1.0f - dirF, 0.8f);
    float pddpf = lm::lm_powf(dirF, 0.8f);
    float pvpf = lm::lm_powf(nclamp(touchVel, 0.0f, kSprintVel), 0.3f);
    float popf = 1.0f - nclamp(posOffset.length(), 0.0f, 0.1f);
    float pf = 1.0f * (0.7f + pddpf * 0.3f) * (0.7f + pvpf * 0.3f) * (0.4f + popf * 0.6f);
    pf = clampf_(pf, 0.0f, 1.0f);
    float adp = 45.0f * (0.7f + lm::lm_powf(oc.touchInfo.desiredPower, 0.5f) * 0.3f);
    float ampf = d.touchMaxPowerFactor;
    if (ampf == 0.0f) ampf = 1.0f;
    float power = clampf_(pf * adp, 0.0f, (32.0f + st(kStPhysicalShotPower) * 13.0f) * (0.2f + ampf * 0.8f));
    float pmbm = (touchMov - bm).length();
    pmbm = nclamp(pmbm, 0.0f, 10.0f);
    power *= 1.0f + pmbm * 0.2f;
    float pdde = lm::lm_powf(dirF, 0.8f);
    float pve = 1.0f - nclamp(fabsf(touchVel - kDribbleVel), 0.0f, 4.0f);
    float poe = 1.0f - nclamp(posOffset.length(), 0.0f, 0.1f);
    float pmbe = 1.0f - pmbm * (0.5f - st(kStTechnicalVolley) * 0.3f);
    float pe = 1.0f - nclamp(power, 30.0f, 100.0f);
    pe = curve(pe, 1.0f);
    float ease = 1.0f * (0.4f + pdde * 0.6f) * (0.7f + pve * 0.3f) * (0.3f + poe * 0.7f) * (0.6f + pmbe * 0.4f) *
                 (0.6f + pe * 0.4f);
    float diff = clampf_(1.0f - ease, 0.0f, 1.0f);
    float desH = 0.05f;
    Vec3 desShot = (oc.touchInfo.desiredDirection.flat() + Vec3(0, 0, desH)).normalized() * power;
    Vec3 worst = oc.touchInfo.desiredDirection.flat();
    float lag = diff * 0.8f;
    worst = (touchDir * lag + worst * (1.0f - lag)).normalized(Vec3(0));
    // GRF evaluates the constructor arguments right to left: z, then y, then x.
    float rz = random_in_range(rng, -1, 1);
    float ry = random_in_range(rng, -1, 1);
    float rx = random_in_range(rng, -1, 1);
    worst = worst + (Vec3(rx, ry, rz) * 0.5f * diff);
    worst.normalize();
    float worstH = curve(lm::lm_powf(diff, 0.7f), 0.7f) * 0.7f;
    float worstP = power * (1.0f - lm::lm_powf(diff, 0.7f) * 0.5f);
    Vec3 worstShot = (worst + Vec3(0, 0, worstH)).normalized() * worstP;
    float wf = random_in_range(rng, 0.0f, 1.0f);
    wf = lm::lm_powf(wf, st(kStTechnicalShot) * 0.7f);
    Vec3 shot = desShot * (1.0f - wf) + worstShot * wf;
    float rcf = 0.3f + wf * 0.7f;
    float pcf = 0.7f;
    xr = -oc.touchInfo.desiredDirection.c[1] * 20.0f + (random_in_range(rng, -20, 20) * rcf);
    yr = -oc.touchInfo.desiredDirection.c[0] * 20.0f + (random_in_range(rng, -20, 20) * rcf);
    float bta = angle2d_to(sp.bodyDirectionVector, shot) / kPi;
    if (fabsf(bta) > 0.5f) bta = (1.0f - fabsf(bta)) * sign_side(bta);
    bta *= 2.0f;
    float amount = bta * 0.25f;
    rot2d_inplace(shot, amount * (0.4f + 0.6f * nclamp(shot.length(), 0.0f, 70.0f)));
    zr = amount * -420 + (random_in_range(rng, -20, 20) * pcf);
    return shot;
}

CB_HDNI Vec3 best_possible_touch(const Sim &s, int p, const Vec3 &desired, int ft) {
    Match &w = s.w;
    Humanoid &h = w.m.players[p].base.humanoid;
    const AnimationState &ca = h.anim;
    const AnimDerived &d = s.D(ca.anim);
    const Vec3 bm = w.m.ball.momentum;
    const float maxShort = 30.0f, maxHigh = 42.0f;
    float base = maxShort;
    if (ft == kFtHighPass) base = maxHigh;
    Vec3 res = desired;
    float mpf = d.touchMaxPowerFactor;
    if (mpf == 0.0f) mpf = 1.0f;
    mpf = mpf * 0.7f + 0.3f;
    float maxPower = base * mpf * (1.0f - clampf_(h.decayingPositionOffset.length() * 2.5f, 0.0f, 0.25f));
    maxPower += bm.length() * 0.5f;
    if (res.length() > maxPower) {
        float missing = res.length() - maxPower;
        res = res.normalized(Vec3(0)) * maxPower;
        res.c[2] += clampf_(missing, 0.0f, 10.0f) * 0.25f;
    }
    float diff = d.touchDifficultyFactor;
    if (ft == kFtShortPass || ft == kFtLongPass) diff *= (1.0f - statistic(s, p, kStTechnicalShortPass) * 0.5f);
    if (ft == kFtHighPass) diff *= (1.0f - statistic(s, p, kStTechnicalHighPass) * 0.5f);
    float df, hf, bmf;
    difficulty_factors(s, p, h.decayingPositionOffset, df, hf, bmf);
    float rr = df * 0.15f + hf * 0.15f + bmf * 0.3f + diff * 0.5f;
    Vec3 abd = rot2d(d.ballDirection, h.startAngle.value() + ca.rotationSmuggleOffset.value());
    if (abd.length() > 0.01f) {
        float bias = clampf_(rr * 1.5f, 0.0f, 1.0f);
        Vec3 native = abd.normalized(res).flat() * res.length() + res * Vec3(0, 0, 1);
        res = res * (1.0f - bias) + native * bias;
    } else {
        float capped = (0.5f < rr) ? 0.5f : rr;
        float rot = random_in_range(w.rng, -0.5f * kPi, 0.5f * kPi) * capped;
        rot2d_inplace(res, rot);
    }
    res *= 1.0f - df * 0.3f;
    res.c[2] += df * 1.5f;
    res.c[2] += bm.c[2] * hf * 0.5f + hf * 1.0f;
    res = res * (1.0f - bmf) + bm * bmf;
    res.c[2] += diff * 5.0f * random_in_range(w.rng, 0.2f, 1.0f);
    return res;
}

}  // namespace cb
