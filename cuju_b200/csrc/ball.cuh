// cuju-b200: ball flight prediction, the time a player needs to reach a point and the earliest
// interception scan.
//   ball_predict_path   GRF Ball::Process prediction; cuju include/cuju/ball.h:30-321
//   time_needed         GRF AI_GetTimeNeededForDistance_ms; cuju include/cuju/ai_time.h:124-231
//   possession_scan     GRF Player::UpdatePossessionStats scan; cuju include/cuju/possession.h:42-120
#pragma once

#include "state.cuh"

namespace cb {

constexpr float kIdleVel = 0.0f, kDribbleVel = 3.5f, kWalkVel = 5.0f, kSprintVel = 8.0f;
constexpr float kAnimSprintVel = 7.0f;
constexpr float kIdleDribbleSwitch = 1.8f, kDribbleWalkSwitch = 4.2f, kWalkSprintSwitch = 6.0f;
constexpr uint32_t kPredictionSpan_ms = 3000;
constexpr uint32_t kCachedPredictions = 100;
constexpr uint32_t kBallHistory = 401;
constexpr uint32_t kTouchOffset_ms = 80;
constexpr float kPitchHalfL = 55, kPitchHalfW = 36;
constexpr float kGoalDepth = 2.55f, kGoalHeight = 2.5f, kGoalHalfW = 3.7f;
constexpr float kLineHalfW = 0.06f;
constexpr float kPlayerHeight = 1.92f;

// A time past the span, or negative (compared unsigned), reads the entry at 2990 ms.
CB_HD Vec3 predict_at(const Vec3 *pred, int t_ms) {
    int i = t_ms;
    if ((uint32_t)i >= kPredictionSpan_ms) i = kPredictionSpan_ms - 10;
    i = i / 10;
    if (i < 0) i = 0;
    return pred[i];
}
CB_HD Vec3 predict_flip(const Vec3 *pred, bool flip, int t_ms) {
    Vec3 p = predict_at(pred, t_ms);
    if (flip) p.mirror();
    return p;
}
CB_HD Vec3 ball_predict(const Ball &b, int t_ms) { return predict_flip(b.predictions, b.lazyFlip, t_ms); }

struct BallMotion {
    Vec3 momentum;
    Quat rotationPerMs;
};

// Post/crossbar bounce against a post center `post` (2-D or XZ) with fallback normal `fb`.
CB_HD void bounce_off(Vec3 &np, const Vec3 &rel, const Vec3 &post, const Vec3 &fb, int keepAxis,
                      Vec3 &normal) {
    const float ballR = 0.11f, postR = 0.07f;
    normal = (rel - post).normalized(fb);
    float kept = np.c[keepAxis];
    np = post + normal * (postR + ballR);
    np.c[keepAxis] = kept;
}

// Fills `predictions` in 10 ms steps (entry k: after 10k ms) and returns the next tick's momentum
// and spin. When the first step lands where the last tick predicted, the previous predictions are
// shifted down instead (at most `validPredictions` ticks in a row).
CB_HDNI void ball_predict_path(Ball &ball, bool ballIsInGoal, BallMotion &out) {
    const float bounce = 0.62f, linearBounce = 0.06f, drag = 0.015f, friction = 0.04f,
                linearFriction = 1.6f, gravity = -9.81f, grassHeight = 0.025f, dt = 0.01f;
    out = BallMotion{};
    Vec3 np = ball.positionBuffer;
    Quat nextOrientation = ball.orientationBuffer;
    Vec3 mom = ball.momentum;
    Quat rot = ball.rotationPerMs;
    ball.predictions[0] = np;
    bool first = true, useCache = false;
    Vec3 ang;
    bool angValid = false;
    auto angles = [&]() {
        if (!angValid) {
            rot.angles(ang.c[0], ang.c[1], ang.c[2]);
            angValid = true;
        }
        return ang;
    };
    ball.touchesNet = false;
    const uint32_t stepMs = (uint32_t)int(dt * 1000.0f);
    for (uint32_t t = stepMs; t < kPredictionSpan_ms + kCachedPredictions * 10; t += stepMs) {
        if (useCache) {
            ball.predictions[t / 10] = ball.predictions[t / 10 + 1];
            continue;
        }
        float frictionFactor = 0.0f;
        mom.c[2] = mom.c[2] + gravity * dt;
        float v = mom.length();
        float vd = v - drag * (v * v) * dt;
        mom = mom.normalized(Vec3(0)) * vd;
        float bottom = np.c[2] - 0.11f;
        float grass = clampf_(1.0f - (bottom / grassHeight), 0.0f, 1.0f);
        grass = lm::lm_powf_pos(grass, 0.7f);
        if (np.c[2] < 0.11f) {
            if (mom.c[2] < 0.0f) {
                frictionFactor = nclamp(-mom.c[2] - 0.5f, 0.0f, 12.0f);
                mom.c[2] = -mom.c[2] * bounce;
                float bv = mom.c[2] - linearBounce;
                mom.c[2] = bv > 0.0f ? bv : 0.0f;
            }
            np.c[2] = 0.11f;
        }
        if (np.c[2] < 0.11f + grassHeight) {
            float af = (friction * grass);
            Vec3 h = mom.flat();
            float hv = h.length();
            float nv = hv - af * (hv * hv) * dt;
            nv = clampf_(nv - (linearFriction * grass * dt), 0.0f, 100000.0f);
            h.normalize(Vec3(0));
            h *= nv;
            mom.c[0] = h.c[0];
            mom.c[1] = h.c[1];
        }
        const float netExp = 2.6f, powerFactor = 1.8f, postAbsorb = 0.8f, ballR = 0.11f,
                    postR = 0.07f, netAbsorb = 0.95f;
        if (first) {
            if (np.c[2] < kGoalHeight + ballR + postR &&
                (np.flat().abs() - Vec3(kPitchHalfL, kGoalHalfW, 0)).length() < ballR + postR) {
                Vec3 normal;
                const float sx = np.c[0] < 0 ? -kPitchHalfL : kPitchHalfL;
                const float sy = np.c[1] < 0 ? -kGoalHalfW : kGoalHalfW;
                const Vec3 fb = np.c[0] < 0 ? Vec3(1, 0, 0) : Vec3(-1, 0, 0);
                bounce_off(np, np.flat(), Vec3(sx, sy, 0), fb, 2, normal);
                mom = (mom.flat().normalized(normal) + (normal * 1.1f)).normalized() *
                          mom.flat().length() * postAbsorb +
                      (Vec3(0, 0, 1) * mom.c[2]);
            }
            Vec3 xz = np * Vec3(1, 0, 1);
            if ((xz.abs() - Vec3(kPitchHalfL, 0, kGoalHeight)).length() < ballR + postR &&
                fabsf(np.c[1]) < kGoalHalfW + ballR + postR) {
                Vec3 normal;
                if (np.c[0] < 0)
                    bounce_off(np, xz, Vec3(-kPitchHalfL, 0, kGoalHeight), Vec3(0, 0, 1), 1, normal);
                else
                    bounce_off(np, xz, Vec3(kPitchHalfL, 0, kGoalHeight), Vec3(0, 0, -1), 1, normal);
                Vec3 mxz = mom * Vec3(1, 0, 1);
                mom = (mxz.normalized(normal) + (normal * 1.1f)).normalized() * mxz.length() *
                          postAbsorb +
                      (Vec3(0, 1, 0) * mom.c[1]);
            }
        }
        if (t <= 10) {
            int inGoal = ballIsInGoal ? 1 : -1;
            bool behind = fabsf(np.c[0]) > kPitchHalfL + 0.11f;
            bool beforeBack = fabsf(np.c[0]) < kPitchHalfL + kGoalDepth - 0.11f;
            bool below = np.c[2] < kGoalHeight + 0.11f;
            bool between = fabsf(np.c[1]) < kGoalHalfW - 0.11f;
            if (ballIsInGoal && !between && behind) {
                float nd = clampf_(fabsf(fabsf(np.c[1]) - kGoalHalfW), 0, 1);
                float power = lm::lm_powf(nd, netExp) * -sign_side(np.c[1]) * inGoal;
                float tension = clampf_((fabsf(mom.c[0]) - kPitchHalfL) * 2.0f, 0.0f, 1.0f);
                float apf = powerFactor + (1.0f - tension) * 3.0f;
                mom.c[1] = mom.c[1] * netAbsorb + power * apf * (100 * dt);
                if (t == 10) ball.touchesNet = true;
            }
            if (ballIsInGoal && !beforeBack && behind) {
                float nd = clampf_(fabsf(fabsf(np.c[0]) - (kPitchHalfL + kGoalDepth)), 0, 1);
                float power = lm::lm_powf(nd, netExp) * -sign_side(np.c[0]) * inGoal;
                mom.c[0] = mom.c[0] * netAbsorb + power * powerFactor * (100 * dt);
                if (t == 10) ball.touchesNet = true;
            }
            if (ballIsInGoal && !below && behind) {
                float nd = clampf_(fabsf(fabsf(np.c[2]) - kGoalHeight), 0, 1);
                float power = lm::lm_powf(nd, netExp) * -inGoal;
                float tension = clampf_((fabsf(mom.c[0]) - kPitchHalfL) * 2.0f, 0.0f, 1.0f);
                float apf = powerFactor + (1.0f - tension) * 3.0f;
                mom.c[2] = mom.c[2] * netAbsorb + power * apf * (100 * dt);
                if (t == 10) ball.touchesNet = true;
            }
        }
        if (np.c[2] < 0.11f + grassHeight) {
            const float radius = 0.11f;
            float avx = mom.c[1] / radius, avy = mom.c[0] / radius;
            Quat rx, ry;
            rx.set_angle_axis(clampf_(avx * 0.001f, -kPi * 0.49f, kPi * 0.49f), Vec3(-1, 0, 0));
            ry.set_angle_axis(clampf_(avy * 0.001f, -kPi * 0.49f, kPi * 0.49f), Vec3(0, 1, 0));
            Quat groundRot = rx * ry;
            Quat o2n = rot.rotation_to(groundRot).normalized();
            float changePerSec = fabsf(o2n.rotation_angle(Quat::identity())) * 1000.0f;
            float maxChange = 1.0f * kPi * grass;
            if (frictionFactor > 0.0f) maxChange += 4.0f * kPi;
            float factor = 1.0f;
            if (changePerSec > maxChange) factor = maxChange / changePerSec;
            if (factor < 1.0f) o2n = o2n.rotation_scaled(factor);
            Quat newRot = o2n * rot;
            const Vec3 a = angles();
            float x = a.c[0], y = a.c[1];
            x = -x;
            Vec3 rm;
            rm.c[0] = y * radius * 1000.0f;
            rm.c[1] = x * radius * 1000.0f;
            float rb = 0.01f;
            rb *= grass;
            if (frictionFactor > 0.0f) rb += 0.5f * frictionFactor;
            rb = clampf_(rb, 0.0f, 1.0f);
            mom.c[0] = mom.c[0] * (1.0f - rb) + rm.c[0] * rb;
            mom.c[1] = mom.c[1] * (1.0f - rb) + rm.c[1] * rb;
            rot = newRot;
            angValid = false;
        }
        {
            Vec3 spin = angles();
            spin *= 10.0f;
            float swerve = nclamp(mom.length(), 0.0f, 70.0f);
            swerve = lm::lm_powf_pos(lm::lm_sinf(swerve * kPi * 0.94f), 2.6f);
            Vec3 am = mom.normalized(Vec3(0)) * swerve * 30.0f;
            Vec3 sw = am.cross(-spin) * 1.0f;
            mom += sw * dt;
        }
        np += mom * dt;
        if (t == 10) {
            Vec3 rv = angles();
            rv *= dt / 0.001f;
            Quat step;
            step.set_angles(rv.c[0], rv.c[1], rv.c[2]);
            nextOrientation = step * nextOrientation;
            out.momentum = mom;
            out.rotationPerMs = rot;
            ball.orientationPrediction = nextOrientation;
            if (ball.validPredictions > 0 && ball.predictions[2] == np) {
                ball.validPredictions--;
                useCache = true;
            } else {
                ball.validPredictions = kCachedPredictions;
            }
        }
        ball.predictions[t / 10] = np;
        first = false;
    }
}

struct TimeNeeded {
    uint32_t usual_ms = 0;
    uint32_t optimistic_ms = 0;
};

CB_HD uint32_t direct_time_ms(const Vec3 &pos, const Vec3 &mov, const Vec3 &target, float maxVel) {
    return (uint32_t)cvt_f_i32(
        roundf((target - (pos + mov * 0.2f)).length() / (maxVel * 0.75f) * 1000));
}

// Usual and optimistic time (ms) a player at `pos` moving with `mov` needs to reach `target`.
// `maxTime_ms` is UINT32_MAX for no limit.
CB_HDNI TimeNeeded time_needed(const Vec3 &pos, const Vec3 &mov, const Vec3 &target, float maxVel,
                               bool precise, uint32_t maxTime_ms) {
    TimeNeeded r;
    const bool limited = maxTime_ms != (uint32_t)-1;
    if ((pos - target).length() > (precise ? 48.0f : 16.0f)) {
        r.usual_ms = direct_time_ms(pos, mov, target, maxVel);
        r.optimistic_ms = r.usual_ms - 200;
        return r;
    }
    Vec3 cur = pos;
    Vec3 cm = mov;
    const float initialOffset = 0.1f;
    if (cm.length() > kIdleDribbleSwitch) {
        cur += cm.normalized() * initialOffset;
        cur += cm * 0.01f;
    } else {
        cur += (target - pos).normalized(Vec3(0)) * initialOffset;
    }
    uint32_t t = 0;
    const uint32_t step = 10;
    float usualR = 0.28f, optR = 0.9f, resultR = usualR;
    bool foundOpt = false;
    const float amv = maxVel * 0.94f;
    while (true) {
        float bias = clampf_((float)t / (float)700, 0, 1);
        if (bias >= 1.0f) {
            float ru = clampf_((target - cur).length() - usualR, 0.0f, 100000.0f);
            r.usual_ms = cvt_f_u32((float)t + (ru / amv) * 1000);
            resultR = usualR + ru;
            if (!foundOpt) {
                float ro = clampf_((target - cur).length() - optR, 0.0f, 100000.0f);
                r.optimistic_ms = cvt_f_u32((float)t + (ro / amv) * 1000);
            }
            break;
        }
        cm.c[0] = mov.c[0] * (1.0f - bias);
        cm.c[1] = mov.c[1] * (1.0f - bias);
        cur.c[0] += cm.c[0] * step * 0.001f;
        cur.c[1] += cm.c[1] * step * 0.001f;
        usualR += amv * bias * step * 0.001f;
        optR += amv * bias * step * 0.001f;
        float d2 = (target - cur).length_sq();
        if ((d2 < optR * optR || (limited && t > maxTime_ms)) && !foundOpt) {
            r.optimistic_ms = t;
            foundOpt = true;
        }
        if (d2 < usualR * usualR || (limited && t > maxTime_ms)) {
            resultR = usualR;
            r.usual_ms = t;
            break;
        }
        t += step;
    }
    if (limited && t > maxTime_ms) {
        uint32_t dt = direct_time_ms(pos, mov, target, maxVel), et = (t + 100) * 2;
        r.usual_ms = dt > et ? dt : et;
        if (!foundOpt) r.optimistic_ms = r.usual_ms;
        return r;
    }
    if (r.usual_ms == 0) {
        r.usual_ms = (uint32_t)cvt_f_i32(
            roundf(clampf_((target - pos).length() / resultR, 0.0f, 1.0f) * 10));
        r.optimistic_ms = r.usual_ms;
    }
    return r;
}

// Earliest times to reach the predicted path of the ball (usual and optimistic), coarse steps sized
// by the ball distance, refined to 10 ms once reachable.
CB_HDNI TimeNeeded possession_scan(const Vec3 *pred, bool flip, const Vec3 &pos, const Vec3 &mov,
                                   float maxVel, bool precise, uint32_t start_ms) {
    TimeNeeded s;
    {
        uint32_t latest = kPredictionSpan_ms;
        uint32_t direct = cvt_f_u32(roundf(
            (predict_flip(pred, flip, kPredictionSpan_ms - 10).flat() - (pos + mov * 0.2f)).length() /
            (maxVel * 0.75f) * 1000));
        s.usual_ms = latest > direct ? latest : direct;
    }
    s.optimistic_ms = s.usual_ms;
    bool refine = false;
    uint32_t stepMs = 10, prev = 0;
    for (uint32_t ms = start_ms; ms < kPredictionSpan_ms; ms += stepMs) {
        if (predict_flip(pred, flip, ms).c[2] < 1.5f) {
            const Vec3 target = predict_flip(pred, flip, ms).flat();
            TimeNeeded r = time_needed(pos, mov, target, maxVel, precise, ms);
            if (r.optimistic_ms <= ms && ms < s.optimistic_ms) s.optimistic_ms = ms;
            if (r.usual_ms <= ms) {
                if (!refine) {
                    ms = prev;
                    stepMs = 10;
                    refine = true;
                } else {
                    s.usual_ms = ms;
                    break;
                }
            }
        }
        if (!refine) {
            float bd = (pos - predict_flip(pred, flip, ms).flat()).length() + 0.2f;
            const float maxBallVel = 50;
            uint32_t ttg = (uint32_t)cvt_f_i32(roundf((bd / maxBallVel) * 1000.0f));
            stepMs = cvt_f_u32(clampf_((float)ttg, 10, 500));
            stepMs = (stepMs / 10) * 10;
        } else {
            stepMs = 10;
        }
        prev = ms;
    }
    return s;
}

}  // namespace cb
