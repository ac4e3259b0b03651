// cuju-b200: world transforms of a humanoid's skeleton nodes and their bounding boxes, and the
// application of one animation frame to the nodes with GRF's smoothing.
//   transforms / boxes   cuju include/cuju/animation/skeleton.h:98-222
//   frame application    cuju include/cuju/animation/apply.h:23-365
#pragma once

#include "match_util.cuh"

namespace cb {

constexpr int kLocalRelative = 0, kLocalAbsolute = 1;

struct Xform {
    Vec3 position, scale;
    Quat rotation;
};
CB_HDNI Xform derive_child(const Xform *parent, int localMode, const Vec3 &pos, const Quat &rot, const Vec3 &scale) {
    Xform d;
    if (localMode == kLocalRelative && parent) {
        d.rotation = (parent->rotation * rot).normalized();
        d.scale = parent->scale * scale;
        d.position = parent->rotation * (parent->scale * pos);
        d.position += parent->position;
    } else {
        d.rotation = rot;
        d.scale = scale;
        d.position = pos;
    }
    return d;
}
CB_HD void derive_nodes(const Skeleton &sk, const NodeState *nodes, Xform out[kNodes]) {
    for (int n = 0; n < sk.nodeCount; n++) {
        const Xform *parent = sk.nodes[n].parent >= 0 ? &out[sk.nodes[n].parent] : nullptr;
        out[n] = derive_child(parent, nodes[n].localMode, nodes[n].position, nodes[n].rotation, nodes[n].scale);
    }
}

struct Aabb {
    Vec3 mn, mx;
    // GRF: the maximum starts at FLT_MIN / 100 (just above zero), so on an axis where every point
    // is negative it stays near zero; collisions depend on it.
    CB_HD void reset() {
        const float smallest = 1.17549435e-38f / 100, largest = 3.40282347e+38f / 100;
        mn.set(largest, largest, largest);
        mx.set(smallest, smallest, smallest);
    }
    CB_HDNI Aabb rotated(const Quat &r) const {
        Vec3 c[8] = {Vec3(mn.c[0], mn.c[1], mn.c[2]), Vec3(mx.c[0], mn.c[1], mn.c[2]),
                     Vec3(mn.c[0], mx.c[1], mn.c[2]), Vec3(mx.c[0], mx.c[1], mn.c[2]),
                     Vec3(mn.c[0], mn.c[1], mx.c[2]), Vec3(mx.c[0], mn.c[1], mx.c[2]),
                     Vec3(mn.c[0], mx.c[1], mx.c[2]), Vec3(mx.c[0], mx.c[1], mx.c[2])};
        Aabb b;
        b.reset();
        for (int i = 0; i < 8; i++) {
            Vec3 v = r * c[i];
            for (int k = 0; k < 3; k++) {
                if (v.c[k] < b.mn.c[k]) b.mn.c[k] = v.c[k];
                if (v.c[k] > b.mx.c[k]) b.mx.c[k] = v.c[k];
            }
        }
        return b;
    }
    CB_HD Aabb translated(const Vec3 &o) const {
        Aabb b = *this;
        b.mn += o;
        b.mx += o;
        return b;
    }
    CB_HDNI bool intersects(const Vec3 &center, float radius) const {
        float d, sq = 0;
        for (int k = 0; k < 3; k++) {
            if (center.c[k] < mn.c[k]) {
                d = center.c[k] - mn.c[k];
                sq += d * d;
            } else if (center.c[k] > mx.c[k]) {
                d = center.c[k] - mx.c[k];
                sq += d * d;
            }
        }
        return sq <= radius * radius;
    }
    // Each coordinate divides by 2 in double.
    CB_HD Vec3 center() const {
        float x = (mn.c[0] + mx.c[0]) / 2.0;
        float y = (mn.c[1] + mx.c[1]) / 2.0;
        float z = (mn.c[2] + mx.c[2]) / 2.0;
        return Vec3(x, y, z);
    }
    // Squares and roots in double (std::pow(float, int)), rounded to float twice.
    CB_HD float radius() const {
        float x = mx.c[0] - mn.c[0], y = mx.c[1] - mn.c[1], z = mx.c[2] - mn.c[2];
        float l = (float)sqrt((double)x * x + (double)y * y);
        return (float)(sqrt((double)l * l + (double)z * z) / 2.0);
    }
};
struct WorldGeom {
    Aabb box;
    Vec3 position;
};
// The mesh box rotated and moved by the world transform (the scale does not enter).
CB_HD WorldGeom geometry_world(const SkelGeometry &g, const Xform &node) {
    Xform d = derive_child(&node, g.localMode, g.position, g.rotation, g.scale);
    Aabb local{g.bbMin, g.bbMax};
    return WorldGeom{local.rotated(d.rotation).translated(d.position), d.position};
}

// ---------------------------------------------------------------------------------------------
// Frame application.
CB_HD float apply_curve(float src, float bias) {
    return (lm::lm_sinf((src - 0.5f) * kPi) * 0.5f + 0.5f) * bias + src * (1.0f - bias);
}
// powf(curve(1 - nclamp(frame, 0, 8), 1), 0.5) for frames 0..8 (clamped).
CB_HD float smooth_begin_bias(int frame) {
    const float t[9] = {0x1p+0f, 0x1.f6297cp-1f, 0x1.d906bep-1f, 0x1.a9b664p-1f, 0x1.6a09e6p-1f,
                        0x1.1c73b4p-1f, 0x1.87de2ap-2f, 0x1.8f8b88p-3f, 0x0p+0f};
    return t[frame < 0 ? 0 : frame > 8 ? 8 : frame];
}
CB_HD int joint_speed_class(int bp) {
    if (bp == kBpLeftElbow || bp == kBpRightElbow || bp == kBpLeftKnee || bp == kBpRightKnee) return 1;
    if (bp == kBpLeftAnkle || bp == kBpRightAnkle) return 2;
    return 0;
}
CB_HD float joint_speed_limit(int cls, float beginBias) {
    float m = 7.5f * kPi;
    if (cls == 1) m *= 1.2f;
    else if (cls == 2) m *= 1.6f;
    return (0.3f + 0.7f * (1.0f - beginBias)) * m;
}
CB_HD float joint_speed(float dot, int dt_ms) {
    return 2.0f * lm::lm_acosf(clampf_(dot, -1.0f, 1.0f)) / ((float)dt_ms * 0.001f);
}

struct ApplyPlan {
    int16_t entry[kBodyParts];
    bool entryNew[kBodyParts];
    float beginBias;
};

// Each node takes the last movement-history entry of its body part, or appends one (node order).
CB_HD bool apply_prepare(const AnimTables &T, const Anim &a, Humanoid &h, bool smooth, int frame, ApplyPlan &plan) {
    plan.beginBias = smooth ? smooth_begin_bias(frame) : 0.0f;
    if (a.nodeCount > kBodyParts) return false;
    if (smooth) {
        auto &mh = h.movementHistory;
        int16_t last[kBodyParts];
        for (int b = 0; b < kBodyParts; b++) last[b] = -1;
        for (int i = 0; i < mh.count; i++) {
            const int32_t bp = mh[i].nodeName;
            if (bp >= 0 && bp < kBodyParts) last[bp] = (int16_t)i;
        }
        for (int n = 0; n < a.nodeCount; n++) {
            const int bp = T.nodes[a.firstNode + n].bodyPart;
            int found = last[bp];
            plan.entryNew[n] = found < 0;
            if (found < 0) {
                if (mh.count >= 32) return false;
                MovementHistoryEntry e;
                memset(&e, 0, sizeof(e));
                e.nodeName = bp;
                e.timeDiff_ms = 10;
                mh[mh.count++] = e;
                found = mh.count - 1;
            }
            plan.entry[n] = (int16_t)found;
        }
    }
    return true;
}

// One node of one humanoid; runs on one lane inside a region.
CB_HDNI void apply_node(const AnimTables &T, const Anim &a, const Skeleton &sk, Humanoid &h, int ni, int frame,
                        bool smooth, float smoothFactor, const Vec3 &basePos, float baseRot, BiasedOffset *offsets,
                        int dt_ms, bool noPosition, const ApplyPlan &plan) {
    const NodeAnim &na = T.nodes[a.firstNode + ni];
    const int bp = na.bodyPart;
    NodeState &node = h.nodes[sk.nodeMap[bp]];
    Quat o;
    Vec3 p;
    {
        Quat o0, o1;
        Vec3 p0, p1;
        float bias = 0.5f;
        node_pose(T, a, na, frame, o0, p0);
        node_pose(T, a, na, frame + 1, o1, p1);
        o0.same_neighborhood(o1);
        o = o0.lerp(bias, o1).normalized();
        p = p0 * (1.0f - bias) + p1 * bias;
    }
    if (bp == kBpPlayer) {
        if (noPosition) {
            p.c[0] = 0;
            p.c[1] = 0;
        } else {
            rot2d_inplace(p, baseRot);
        }
    }
    if (bp == kBpBody) {
        Quat rz;
        rz.set_angle_axis(baseRot, Vec3(0, 0, 1));
        o = rz * o;
        o.normalize();
    }
    {
        BiasedOffset &off = offsets[bp];
        if (off.bias != 0.0) {
            off.orientation.same_neighborhood(o);
            o = o.lerp(off.bias, off.orientation).normalized();
        }
    }
    if (smooth) {
        MovementHistoryEntry *e = &h.movementHistory[plan.entry[ni]];
        if (plan.entryNew[ni]) {
            e->position = p;
            e->orientation = o;
        }
        const float beginBias = plan.beginBias;
        float curBias = 0.0f + beginBias * smoothFactor * 0.5f;
        if (bp != kBpPlayer) {
            const Quat prev = e->orientation;
            Quat cur = node.rotation;
            cur.same_neighborhood(prev);
            if (dt_ms > 0) {
                o = o.slerp(curBias, cur).normalized();
                float dot = o.same_neighborhood(cur);
                const float maxAngle = joint_speed_limit(joint_speed_class(bp), beginBias);
                float aps = joint_speed(dot, dt_ms);
                if (aps > maxAngle) {
                    float frac = maxAngle / aps;
                    Quat desired = cur.rotation_to(o).normalized();
                    o = (desired.rotation_scaled(frac) * cur).normalized();
                }
            }
            e->orientation = cur;
            e->timeDiff_ms = dt_ms;
        } else {
            const Vec3 curPos = node.position;
            if (dt_ms > 0 && beginBias > 0.01f) {
                p.c[2] = p.c[2] * (1.0f - curBias) + curPos.c[2] * curBias;
                float maxMps = 2.8f;
                if (a.outgoingSpecialState != kSS_Empty) maxMps = 6.0f;
                float allowed = maxMps * ((float)dt_ms * 0.001f);
                float newZ = p.c[2] + basePos.c[2];
                float desired = fabsf(newZ - curPos.c[2]);
                float hb = 1.0f;
                if (desired > allowed) hb = allowed / desired;
                newZ = (newZ * hb + curPos.c[2] * (1.0f - hb)) * beginBias + newZ * (1.0f - beginBias);
                p = p.flat() + Vec3(0, 0, newZ);
            }
            e->position = curPos;
            e->timeDiff_ms = dt_ms;
        }
    }
    if (bp != kBpPlayer) {
        Quat cur = node.rotation;
        o.same_neighborhood(cur);
        node.rotation = o;
    } else {
        node.position = p + basePos;
    }
}

}  // namespace cb
