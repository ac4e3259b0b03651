// cuju-b200: referee and linesmen, force fields, offside lines from mental images, pose offsets
// of moving players, and the in-game camera (whose shake draws from the match RNG).
//   officials / force fields / offside  cuju include/cuju/simulation/officials.h:19-396
//   geometry offsets                    cuju include/cuju/simulation/geometry_offsets.h:14-197
//   camera                              cuju include/cuju/simulation/camera.h:18-167
#pragma once

#include "humanoid.cuh"

namespace cb {

constexpr float kDistToVel = 2.6f;
constexpr float kBallDistOptimize = 10.0f;
enum MagnetType { kAttract, kRepel };
enum DecayType { kDecayConstant, kDecayVariable };

struct ForceSpot {
    Vec3 origin;
    int magnetType = kAttract;
    int decayType = kDecayConstant;
    float exponent = 1.0f;
    float power = 0.0f;
    float scale = 0.0f;
};
using ForceField = List<ForceSpot, 64>;

CB_HD bool field_push(const Sim &s, ForceField &f, const ForceSpot &sp) {
    if (f.count >= 64) return s.fail(kStatusOverflow);
    f.push(sp);
    return true;
}

// The spot terms are computed in parallel and summed in spot order.
CB_HDNI Vec3 force_field_movement(const ForceField &f, const Vec3 &pos, float dampDist = 10) {
    Vec3 cv;
    float cf = 0.0f;
    struct Term {
        Vec3 contribution;
        float force;
        int32_t active;
    };
    auto term = [&](int i) {
        const ForceSpot &sp = f[i];
        Term t{Vec3(), 0.0f, 0};
        float d = (sp.origin - pos).length();
        float in;
        if (sp.decayType == kDecayConstant) {
            in = 1.0f;
        } else {
            in = clampf_(1.0f - d / sp.scale, 0.0f, 1.0f);
            if (sp.exponent != 1.0f) in = lm::lm_powf(in, sp.exponent);
        }
        if (in > 0.0f) {
            Vec3 rel = sp.origin - pos;
            rel.normalize(Vec3(0));
            if (sp.magnetType == kRepel) rel = -rel;
            else if (d < dampDist) rel *= d / dampDist;
            float force = sp.power * in;
            t.contribution = rel * force;
            t.force = force;
            t.active = 1;
        }
        return t;
    };
    crew_pipeline<Term>(f.count, term, [&](int, const Term &t) {
        if (t.active) {
            cv += t.contribution;
            cf += t.force;
        }
    });
    if (cf == 0.0f) return Vec3(0);
    return (cv / cf) * kSprintVel;
}

struct ImagePos {
    Vec3 position, movement;
    int role;
};
using ImageList = List<ImagePos, kPlayers>;

// The active players of a team as a mental image sees them, extrapolated and clamped to reality;
// in the image's order.
CB_HDNI void mental_team_images(const Match &w, int mi, int teamID, ImageList &out) {
    const MentalImage &im = w.m.mentalImages[mi];
    const int age = (int)(w.m.actualTime_ms - (uint64_t)im.timeStamp_ms);
    out.count = 0;
    struct Entry {
        Vec3 position, movement;
        int32_t role, valid;
    };
    auto img = [&](int i) {
        const PlayerImage &pi = im.players[i];
        Entry e{Vec3(), Vec3(), 0, 0};
        if (!w.m.players[pi.player].base.isActive || w.playerTeamID[pi.player] != teamID) return e;
        const SpatialState &sp = hum(w, pi.player).spatial;
        Vec3 extr = pi.movement * (float)age * 0.001f;
        Vec3 p = pi.position + extr;
        e.position = p.max_deviation(sp.position, im.maxDistanceDeviation);
        e.movement = pi.movement.max_deviation(sp.movement, im.maxMovementDeviation);
        e.role = pi.role;
        e.valid = 1;
        return e;
    };
    crew_pipeline<Entry>(im.players.count, img, [&](int, const Entry &e) {
        if (e.valid) out.push(ImagePos{e.position, e.movement, e.role});
    });
}
// Moves each image ahead along x by `future_ms`, in place.
CB_HDNI float offside_line_from_images(ImageList &im, const Vec3 &ball, int side, unsigned int future_ms) {
    int ignored = 0;
    Vec3 deepest;
    for (int i = 0; i < im.count; i++) {
        im[i].position.c[0] += im[i].movement.c[0] * future_ms * 0.001f;
        if (im[i].position.c[0] * side > im[ignored].position.c[0] * side) ignored = i;
    }
    for (int i = 0; i < im.count; i++) {
        if (im[i].position.c[0] * side > deepest.c[0] * side && i != ignored) deepest = im[i].position;
    }
    float line = deepest.c[0];
    if (ball.c[0] * side > line * side) line = ball.c[0];
    if (line * side < 0) line = 0;
    return clampf_(line, -kPitchHalfL, kPitchHalfL);
}
CB_HD float offside_line(const Match &w, int mi, int teamID, unsigned int future_ms = 0) {
    ImageList im;
    mental_team_images(w, mi, teamID, im);
    return offside_line_from_images(im, mental_ball(w, mi, 0), team_side(w, teamID), future_ms);
}
CB_HDNI Vec3 ball_average_position(const Match &w, unsigned int dur_ms) {
    const Ball &b = w.m.ball;
    unsigned int total = 0;
    Vec3 avg;
    for (int i = b.positionHistory.count - 1; i >= 0; i--) {
        Vec3 p = b.positionHistory[i];
        if (b.lazyFlip) p.mirror();
        avg += p;
        total++;
        if (total * 10 > dur_ms) break;
    }
    if (total > 0) avg /= Vec3((float)total);
    else avg = ball_predict(b, 0);
    return avg;
}

CB_HDNI void referee_request_command(const Sim &s, int official, CommandQueue &q) {
    Match &w = s.w;
    const MatchState &m = w.m;
    const SpatialState &sp = m.officials[official].humanoid.spatial;
    const Vec3 pos = sp.position;
    if (official == 0) {
        const Referee &ref = m.referee;
        if (ref.buffer.active && (ref.foul.foulType == 2 || ref.foul.foulType == 3) &&
            ref.buffer.prepareTime > m.actualTime_ms + 5000) {
            const Vec3 offender = hum(w, ref.foul.foulPlayer).spatial.position;
            Vec3 des = offender + (pos - offender).normalized(Vec3(0)) * (float)2.0;
            if ((double)(pos - des).length() > 2.0) {
                PlayerCommand c;
                default_command(c);
                c.desiredFunctionType = kFtMovement;
                c.useDesiredMovement = true;
                c.useDesiredLookAt = true;
                c.desiredDirection = (des - pos).normalized(sp.directionVector);
                c.desiredVelocityFloat = range_velocity((des - pos).length() * 1.0f);
                c.desiredLookAt = offender;
                queue_push(s, q, c);
            } else {
                PlayerCommand c;
                default_command(c);
                c.desiredFunctionType = kFtSpecial;
                c.useDesiredMovement = false;
                c.useDesiredLookAt = false;
                c.useSpecialVar1 = true;
                c.specialVar1 = 3;
                queue_push(s, q, c);
                PlayerCommand f;
                default_command(f);
                f.desiredFunctionType = kFtMovement;
                f.useDesiredMovement = true;
                f.useDesiredLookAt = true;
                f.desiredDirection = (des - pos).normalized(sp.directionVector);
                f.desiredVelocityFloat = kIdleVel;
                f.desiredLookAt = offender;
                queue_push(s, q, f);
            }
        } else {
            PlayerCommand c;
            default_command(c);
            c.desiredFunctionType = kFtMovement;
            c.useDesiredMovement = true;
            c.useDesiredLookAt = true;
            ForceField ff;
            {
                ForceSpot sp0;
                sp0.origin = ball_average_position(w, 2000).flat() * 0.6f;
                sp0.magnetType = kAttract;
                sp0.decayType = kDecayConstant;
                sp0.power = 0.5f;
                field_push(s, ff, sp0);
            }
            {
                ForceSpot sp1;
                sp1.origin = ball_at(w, 200).flat();
                sp1.magnetType = kRepel;
                sp1.decayType = kDecayVariable;
                sp1.power = 0.5f;
                sp1.scale = 10.0f;
                field_push(s, ff, sp1);
            }
            const int teams[2] = {w.firstTeamID(), 1 - w.firstTeamID()};
            for (int t = 0; t < 2; t++) {
                PlayerList ap;
                active_players(ap, w, teams[t]);
                for (int i = 0; i < ap.count; i++) {
                    const SpatialState &ps = hum(w, ap[i]).spatial;
                    ForceSpot spx;
                    spx.origin = ps.position + ps.movement * 0.4f;
                    spx.magnetType = kRepel;
                    spx.decayType = kDecayVariable;
                    spx.power = 0.5f;
                    spx.scale = 10.0f;
                    field_push(s, ff, spx);
                }
            }
            Vec3 des = pos + force_field_movement(ff, pos);
            c.desiredDirection = (des - pos).normalized(sp.directionVector);
            c.desiredVelocityFloat = clampf_((des - pos).length() * kDistToVel * 0.5f, kIdleVel, kSprintVel);
            c.desiredLookAt = ball_at(w, 60).flat();
            queue_push(s, q, c);
        }
    } else {
        PlayerCommand c;
        default_command(c);
        c.desiredFunctionType = kFtMovement;
        c.useDesiredMovement = true;
        c.useDesiredLookAt = true;
        float line;
        Vec3 des;
        const int latest = mental_index(w, 0);
        if (pos.c[1] < 0) {
            line = offside_line(w, latest, 1);
            des = Vec3(line, -(kPitchHalfW + 0.8f), 0);
        } else {
            line = offside_line(w, latest, 0);
            des = Vec3(line, kPitchHalfW + 0.8f, 0);
        }
        c.desiredDirection = (des - pos).normalized(sp.directionVector);
        c.desiredVelocityFloat = range_velocity((des - pos).length() * kDistToVel);
        c.desiredLookAt = Vec3(des.c[0], 0, 0);
        queue_push(s, q, c);
    }
}

// The interrupt branch of an official's tick: the referee's command and the animation selection.
// Reads and writes only the match, so a whole warp can run it for one environment.
CB_HDNI bool official_interrupt(const Sim &s, int official) {
    const int hi = s.w.m.playerCount + official;
    Humanoid &h = s.w.m.officials[official].humanoid;
    AnimationState &ca = h.anim;
    CommandQueue q;
    if (h.interruptAnim == kIntTrip && h.tripType != 0) {
        add_trip_commands(s, h, q, h.tripType);
        h.tripType = 0;
        PlayerCommand bmc;
        basic_movement_command(bmc, h, h.spatial.floatVelocity);
        queue_push(s, q, bmc);
    } else {
        referee_request_command(s, official, q);
    }
    bool found = false;
    for (int i = 0; i < q.count; i++) {
        Selector sel(s, hi);
        int r = sel.base_select(q[i], h.interruptAnim);
        if (r == kSelUnsupported) return s.fail(kStatusUnsupported);
        if (*s.status != kStatusOk) return false;
        found = r == kSelTrue;
        if (found) break;
    }
    if (found) {
        h.startPosition = h.spatial.position;
        h.startAngle = h.spatial.angle;
        {
            Selector sel(s, hi);
            Vec3 nsp;
            float nsa;
            sel.predicted_situation(nsp, nsa);
            h.nextStartPosition = nsp;
            set_radian(h.nextStartAngle, nsa);
        }
        h.applyBuffer.anim = ca.anim;
        h.applyBuffer.smooth = true;
        h.applyBuffer.smoothFactor = (h.interruptAnim == kIntSwitch) ? 0.6f : 1.0f;
        float ad = s.D(ca.anim).animDifficultyFactor;
        if (ad > h.decayingDifficultyFactor) h.decayingDifficultyFactor = ad;
        if (h.interruptAnim == kIntReQueue && h.prevAnimFunctionType == ca.functionType) h.requeueDelayFrames = 32;
    }
    return true;
}

CB_HDNI bool official_process(const Sim &s, int official) {
    Match &w = s.w;
    Humanoid &h = w.m.officials[official].humanoid;
    AnimationState &ca = h.anim;
    h.decayingPositionOffset *= 0.95f;
    if ((double)h.decayingPositionOffset.length() < 0.005) h.decayingPositionOffset = Vec3(0);
    h.decayingDifficultyFactor = clampf_(h.decayingDifficultyFactor - 0.002f, 0.0f, 1.0f);
    calc_spatial_state(s, h);
    h.spatial.positionOffsetMovement = Vec3(0);
    ca.frameNumber++;
    h.prevAnimFrameNumber++;
    if (ca.frameNumber == s.A(ca.anim).frameCount - 1 && h.interruptAnim == kIntNone) h.interruptAnim = kIntSwitch;
    if (!crew_assist(s, kJobOfficialInterrupt, official, h.interruptAnim != kIntNone)) return false;
    h.requeueDelayFrames = (int)clampf_((float)(h.requeueDelayFrames - 1), 0, 10000);
    h.interruptAnim = kIntNone;
    const Anim &pa = s.A(ca.anim);
    float fb = (ca.frameNumber + 1) / (float)((pa.frameCount - 1) + 1);
    set_radian(ca.rotationSmuggleOffset, ca.rotationSmuggle.begin.value() * (1.0f - fb) + ca.rotationSmuggle.end.value() * fb);
    h.applyBuffer.frameNumber = ca.frameNumber;
    if ((uint32_t)ca.positions.count > (uint32_t)ca.frameNumber) {
        h.applyBuffer.position = h.startPosition + ca.actionSmuggleOffset + ca.actionSmuggleSustainOffset +
                                 ca.movementSmuggleOffset + ca.positions[ca.frameNumber];
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
// The branches the lanes of a warp share in assist rounds (assist.cuh: crew_assist).
CB_HDNI bool assist_job(const Sim &s, int kind, int arg) {
    switch (kind) {
        case kJobInterrupt: return humanoid_interrupt(s, arg);
        case kJobTouches: return humanoid_touches(s, arg);
        case kJobOfficialInterrupt: return official_interrupt(s, arg);
        default: return s.fail(kStatusUnsupported);
    }
}

CB_HD bool officials_process(const Sim &s) {
    for (int o = 0; o < 3; o++)
        if (!official_process(s, o)) return false;
    return true;
}

// ---------------------------------------------------------------------------------------------
// Pose offsets (GRF PlayerBase::CalculateGeometryOffsets).
CB_HD void set_offset(Humanoid &h, int bp, float bias, const Quat &o) {
    h.offsets[bp].bias = bias;
    h.offsets[bp].orientation = o;
}
CB_HDNI int team_best_possession_player(const Match &w, int teamID) {
    int bt = 10000000, bp = -1;
    for (int p = 0; p < w.m.playerCount; p++) {
        if (w.playerTeamID[p] != teamID || !w.m.players[p].base.isActive) continue;
        int t = (int)w.m.players[p].timeNeededToGetToBall_ms;
        if (t < bt) {
            bt = t;
            bp = p;
        }
    }
    return bp;
}
// Runs on one lane (inside a region); writes only player p.
CB_HDNI void geometry_offsets(const Sim &s, int p) {
    Match &w = s.w;
    Humanoid &h = w.m.players[p].base.humanoid;
    const SpatialState &sp = h.spatial;
    const Quat ident(0, 0, 0, 1);
    for (int bp = kBpMiddle; bp <= kBpBody; bp++) set_offset(h, bp, 0.0, ident);
    const float legInfluence = 0.7f, bodyInfluence = 0.5f, armInfluence = 0.9f;
    if (!(w.m.inPlay && w.m.ballRetainer != p)) return;
    if (h.anim.functionType != kFtMovement) return;
    {
        float av = sp.actualMovement.length();
        float anv = sp.animationMovement.length();
        float vf = (av + 0.2f) / (anv + 0.2f);
        float faster = 0.0f;
        if (sp.actualMovement.length() > 7.0f) faster += 0.1;
        vf = clampf_(vf, 0.1f, 1.0f + faster);
        float bend = 0.8f;
        Quat lh = angle_axis_quat(-0.15f * kPi * bend, Vec3(1, 0.06, -0.12).normalized());
        Quat rh = angle_axis_quat(-0.15f * kPi * bend, Vec3(1, -0.06, 0.12).normalized());
        Quat knee = angle_axis_quat(0.3f * kPi * bend, Vec3(1, 0, 0));
        Quat ankle = angle_axis_quat(-0.1f * kPi * bend, Vec3(1, 0, 0));
        float lb = (1.0f - vf) * legInfluence;
        set_offset(h, kBpLeftThigh, lb, lh);
        set_offset(h, kBpRightThigh, lb, rh);
        set_offset(h, kBpLeftKnee, lb, knee);
        set_offset(h, kBpRightKnee, lb, knee);
        set_offset(h, kBpLeftAnkle, lb, ankle);
        set_offset(h, kBpRightAnkle, lb, ankle);
    }
    if (!w.m.players[p].hasPossession) {
        Vec3 toBall = (mental_ball(w, mental_index(w, h.mentalImageTime), 10).flat() - sp.position)
                          .normalized(sp.directionVector);
        float angle = angle2d_to(toBall, rot2d(sp.relBodyDirectionVectorNonQuantized, sp.angle.value()));
        angle = clampf_(fabsf(angle) - 0.05f * kPi, 0.0f, kPi) * sign_side(angle);
        float lab = lm::lm_powf(1.0f - fabsf(angle / kPi), 0.3f);
        lab = clampf_(lab * bodyInfluence, 0.0f, 1.0f);
        float bd = get_distance(ball_at(w, 100).flat(), sp.position);
        float fall = 1.6f;
        if (bd < fall) lab *= nclamp(bd, fall * 0.4f, fall);
        float vfr = nclamp(sp.floatVelocity, kIdleVel, kSprintVel - 0.5f);
        lab *= 1.0f - vfr * vfr * 0.3f;
        Quat mid = angle_axis_quat(angle, Vec3(0, 0, 1));
        mid.normalize();
        set_offset(h, kBpMiddle, lab * 0.3f, mid);
        Quat head = angle_axis_quat(angle, Vec3(0, 0, 1));
        head.normalize();
        set_offset(h, kBpNeck, lab * 0.7f, head);
    }
    {
        const int teamID = w.playerTeamID[p];
        int opp = team_best_possession_player(w, 1 - teamID);
        if (opp < 0) {
            s.fail(kStatusUnsupported);
            return;
        }
        const SpatialState &os = hum(w, opp).spatial;
        if ((double)(os.position - sp.position).length() < 1.4 && (double)os.directionVector.dot(sp.directionVector) > 0.0) {
            Vec3 base = rot2d(rot2d(Vec3(0, -1, 0), sp.angle.value()), sp.relBodyAngle.value());
            Vec3 ov = os.position - sp.position;
            float angle = angle2d_to(base, ov.normalized(base));
            const double aa = fabsf(angle);
            const double dpi = (double)kPi;
            if (aa > 0.6 * dpi && aa < 0.85 * dpi) {
                Quat sh, el;
                if (angle > 0) {
                    sh = angle_axis_quat((float)(0.4 * dpi), Vec3(0, 1, 0));
                    el = angle_axis_quat(0, Vec3(0, 1, 0));
                    set_offset(h, kBpRightShoulder, 0.8f * armInfluence, sh.normalized());
                    set_offset(h, kBpRightElbow, 0.7f * armInfluence, el.normalized());
                } else {
                    sh = angle_axis_quat((float)(-0.4 * dpi), Vec3(0, 1, 0));
                    el = angle_axis_quat(0, Vec3(0, 1, 0));
                    set_offset(h, kBpLeftShoulder, 0.8f * armInfluence, sh.normalized());
                    set_offset(h, kBpLeftElbow, 0.7f * armInfluence, el.normalized());
                }
                Quat mid = angle_axis_quat(0.2f * kPi, Vec3(1, 0, 0));
                set_offset(h, kBpMiddle, 0.3f * armInfluence, mid.normalized());
            }
            if (aa > 0.2 * dpi && aa <= 0.6 * dpi) {
                Quat sh, el;
                if (angle > 0) {
                    sh = angle_axis_quat((float)(0.4 * dpi), Vec3(0, 1, 0));
                    el = angle_axis_quat((float)(-0.5 * dpi), Vec3(1, 0, 0));
                    set_offset(h, kBpRightShoulder, 0.7f * armInfluence, sh.normalized());
                    set_offset(h, kBpRightElbow, 0.8f * armInfluence, el.normalized());
                } else {
                    sh = angle_axis_quat((float)(-0.4 * dpi), Vec3(0, 1, 0));
                    el = angle_axis_quat((float)(-0.5 * dpi), Vec3(1, 0, 0));
                    set_offset(h, kBpLeftShoulder, 0.7f * armInfluence, sh.normalized());
                    set_offset(h, kBpLeftElbow, 0.8f * armInfluence, el.normalized());
                }
            }
            // GRF: this bound is 0.2 radians, not 0.2 * pi.
            if (aa < 0.2) {
                Quat sh = angle_axis_quat((float)(-0.4 * dpi), Vec3(1, 0, 0));
                Quat el = angle_axis_quat((float)(-0.2 * dpi), Vec3(1, 0, 0));
                if (angle > 0) {
                    set_offset(h, kBpRightShoulder, 0.6f * armInfluence, sh.normalized());
                    set_offset(h, kBpRightElbow, 0.8f * armInfluence, el.normalized());
                } else {
                    set_offset(h, kBpLeftShoulder, 0.6f * armInfluence, sh.normalized());
                    set_offset(h, kBpLeftElbow, 0.8f * armInfluence, el.normalized());
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Camera.
constexpr float kCamZoom = 0.5f, kCamHeight = 0.3f, kCamFov = 0.4f, kCamAngleFactor = 0.0f;
constexpr unsigned int kCamPositions = 150;
CB_HD float camera_weight(int i, int n) {
    const float sz = n;
    float wgt = lm::lm_sinf((i / sz - 0.3f) * 1.4f * kPi) * 0.5f + 0.5f;
    wgt *= lm::lm_powf(1.0f - i / sz, 0.3f);
    return wgt;
}
CB_HDNI void update_ingame_camera(const Sim &s) {
    Match &w = s.w;
    MatchState &m = w.m;
    const int first = w.firstTeamID(), second = 1 - first;
    float fov = 0.5f + kCamFov * 0.5f;
    float zoom = kCamZoom;
    float height = kCamHeight * 1.5f;
    float playerBias = 0.6f;
    const SpatialState &ds = hum(w, m.designatedPossessionPlayer).spatial;
    Vec3 bp = ball_predict(m.ball, 0) * (1.0f - playerBias) + ds.position * playerBias;
    bp += ds.directionVector * 1.0f;
    bp += Vec3(((team_by_id(w, first).fadingTeamPossessionAmount - 1.0f) * -team_side(w, first) +
                (team_by_id(w, second).fadingTeamPossessionAmount - 1.0f) * -team_side(w, second)) *
                   4.0f,
               0, 0);
    bp.c[2] *= 0.1f;
    float mw = (float)((double)(kPitchHalfL * 0.84f) * (1.0 / (double)(zoom + 0.01f)));
    float mh = (float)((double)(kPitchHalfW * 0.60f) * (1.0 / (double)(zoom + 0.01f)) * (double)(height * 0.75f + 0.25f));
    if (fabsf(bp.c[0]) > mw) bp.c[0] = mw * sign_side(bp.c[0]);
    if (fabsf(bp.c[1]) > mh) bp.c[1] = mh * sign_side(bp.c[1]);
    // GRF evaluates the constructor arguments right to left: y draws before x.
    float ry = random_in_range(w.rng, -0.1f, 0.1f);
    float rx = random_in_range(w.rng, -0.1f, 0.1f);
    Vec3 shudder = Vec3(rx, ry, 0) * (m.ball.momentum.length() * 0.8f + 6.0f);
    shudder *= 0.2f;
    auto &cp = m.cameraPosition;
    Vec3 add = bp + shudder * ((float)cp.count / (float)kCamPositions);
    if (cp.count == (int)kCamPositions) {
        for (int i = 0; i + 1 < cp.count; i++) cp[i] = cp[i + 1];
        cp[cp.count - 1] = add;
    } else {
        cp[cp.count++] = add;
    }
    Vec3 avg;
    float cnt = 0;
    const int n = cp.count;
    const float *table = s.ctx.cameraWeights ? s.ctx.cameraWeights + n * (n - 1) / 2 : nullptr;
    for (int i = 0; i < n; i++) {
        float wgt = table ? table[i] : camera_weight(i, n);
        avg += cp[i] * wgt;
        cnt += wgt;
    }
    avg /= Vec3(cnt);
    float af = 1.0f - kCamAngleFactor * 0.4f;
    if (!m.goalScored || (m.goalScored && m.goalScoredTimer < 1000)) {
        zoom = (0.6f + zoom * 1.0f) * (1.0f / fov);
        height = 4.0f + height * 10;
        float dr = avg.c[1] / 800.0f;
        m.cameraOrientation.set_angle_axis(dr + (0.42f - height * 0.01f) * kPi, Vec3(1, 0, 0));
        m.cameraNodeOrientation.set_angle_axis((-avg.c[0] / kPitchHalfL) * (1.0f - af) * 0.25f * kPi * 1.24f,
                                               Vec3(0, 0, 1));
        m.cameraNodePosition =
            avg * Vec3(1.0f * (1.0f - kCamAngleFactor * 0.2f) * (1.0f - kCamZoom * 0.3f), 0.9f - kCamZoom * 0.3f, 0.2f) +
            Vec3(0, -41.4f - (kCamFov * 3.7f) + lm::lm_powf(height, 1.2f) * 0.46f, 10.0f + height) * zoom;
        m.cameraFieldOfView = (fov * 28.0f) - (m.cameraNodePosition.c[1] / 30.0f);
        m.cameraNearCap = m.cameraNodePosition.c[2];
        m.cameraFarCap = 200;
    } else {
        Vec3 target = ball_predict(m.ball, 0).flat();
        if (m.lastGoalScorer >= 0) target = hum(w, m.lastGoalScorer).spatial.position;
        float rot = (float)m.goalScoredTimer * 0.0005f;
        m.cameraOrientation.set_angle_axis(0.45f * kPi, Vec3(1, 0, 0));
        m.cameraNodeOrientation.set_angle_axis(rot, Vec3(0, 0, 1));
        m.cameraNodePosition = target + rot2d(Vec3(0, -1, 0), rot) * 15.0f + Vec3(0, 0, 3);
        m.cameraFieldOfView = 35.0f;
        m.cameraNearCap = 1;
        m.cameraFarCap = 220;
    }
}
// The camera works on the unmirrored pitch, so team 1 is mirrored around its update.
CB_HDNI void update_camera(const Sim &s) {
    Match &w = s.w;
    MatchState &m = w.m;
    if (m.autoUpdateInGameCamera) {
        mirror_match(w, false, true, false);
        update_ingame_camera(s);
        mirror_match(w, false, true, false);
    }
    unsigned int zoomTime = 2000, startTime = 0;
    if (m.actualTime_ms < zoomTime + startTime) {
        Quat init(0, 0, 0, 1);
        init.set_angle_axis(0.0f * kPi, Vec3(1, 0, 0));
        Quat heading(0, 0, 0, 1);
        init = heading * init;
        Vec3 initPos = Vec3(0.0f, 0.0f, 60.0);
        int el = cvt_f_i32(clampf_((float)(m.actualTime_ms - startTime), 0, zoomTime));
        float bias = el / (float)(zoomTime);
        bias *= kPi;
        bias = lm::lm_sinf(bias - 0.5f * kPi) * -0.5f + 0.5f;
        m.cameraOrientation = m.cameraOrientation.slerp(bias, Quat(0, 0, 0, 1));
        m.cameraNodeOrientation = m.cameraNodeOrientation.slerp(bias, init);
        m.cameraNodePosition = m.cameraNodePosition * (1.0f - bias) + initPos * bias;
        m.cameraFieldOfView = m.cameraFieldOfView * (1.0f - bias) + 40 * bias;
        m.cameraNearCap = m.cameraNearCap * (1.0f - bias) + 2.0f * bias;
    }
}

}  // namespace cb
