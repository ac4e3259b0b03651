// cuju-b200: animation selection of players and officials: a crude filter over the animation
// table (lane-parallel ballot compaction), chained stable sorts (bitonic sort of (key, position)
// pairs in the warp's scratch, which equals a stable sort for NaN-free keys) and the physics
// vector that turns an animation into positions.
// GRF's selection: cuju include/cuju/simulation/select_animation.h (crude filter :568-810,
// sort keys :812-933, Selector :935-2188, BaseSelectAnimation :2189-2336, SelectAnimation
// :2338-2792). Every expression keeps GRF's operation order, precision and conversions.
#pragma once

#include "match_util.cuh"

namespace cb {

enum SelectResult { kSelFalse = 0, kSelTrue = 1, kSelUnsupported = 2 };
constexpr int kMaxAnims = 1536;
using AnimList = List<int16_t, kMaxAnims>;
using PosList = List<Vec3, kAnimPositions>;

CB_HD int velocity_id(int v, bool dribbleAsWalk = false) {
    int id = 0;
    switch (v) {
        case kVelIdle: id = 0; break;
        case kVelDribble: id = 1; break;
        case kVelWalk: id = 2; break;
        case kVelSprint: id = 3; break;
        default: id = 0; break;
    }
    if (dribbleAsWalk && id > 1) id--;
    return id;
}
CB_HD float curve(float src, float bias = 1.0f) {
    return (lm::lm_sinf((src - 0.5f) * kPi) * 0.5f + 0.5f) * bias + src * (1.0f - bias);
}
CB_HD void normalize_to(Vec3 &v, float len) {
    float f = len / sqrtf(v.dot(v));
    v.c[0] *= f;
    v.c[1] *= f;
    v.c[2] *= f;
}
CB_HD Vec3 normalized_to(const Vec3 &v, float len) { Vec3 r = v; normalize_to(r, len); return r; }
CB_HD void normalize_max(Vec3 &v, float len) {
    if (v.length() > len) {
        v.normalize();
        v *= len;
    }
}
CB_HD Vec3 normalized_max(const Vec3 &v, float len) {
    if (v.length() > len) return v.normalized(Vec3(0)) * len;
    return v;
}
// Float differences whose squares sum in double.
CB_HD float get_distance(const Vec3 &a, const Vec3 &b) {
    float dx = a.c[0] - b.c[0], dy = a.c[1] - b.c[1], dz = a.c[2] - b.c[2];
    if (dx == 0.0f && dy == 0.0f && dz == 0.0f) return 0.0f;
    double x = dx, y = dy, z = dz;
    float l = (float)sqrt(x * x + y * y + z * z);
    if (l < kAboveMicro) l = 0;
    return l;
}

// 11 preferred directions: angles are double products with pi rounded to float.
CB_HD float preferred_angle(int i) {
    const double f[11] = {0, 0.111, -0.111, 0.25, -0.25, 0.5, -0.5, 0.75, -0.75, 0.999, -0.999};
    return (float)(f[i] * (double)kPi);
}
// Vec3(0,-1,0) rotated by each preferred angle (the vector itself for angle 0).
CB_HD Vec3 preferred_dir(int i) {
    switch (i) {
        case 0: return Vec3(0x0p+0f, -0x1p+0f, 0x0p+0f);
        case 1: return Vec3(0x1.5de48ap-2f, -0x1.e12f08p-1f, 0x0p+0f);
        case 2: return Vec3(-0x1.5de48ap-2f, -0x1.e12f08p-1f, 0x0p+0f);
        case 3: return Vec3(0x1.6a09e6p-1f, -0x1.6a09e6p-1f, 0x0p+0f);
        case 4: return Vec3(-0x1.6a09e6p-1f, -0x1.6a09e6p-1f, 0x0p+0f);
        case 5: return Vec3(0x1p+0f, 0x1.777a5cp-25f, 0x0p+0f);
        case 6: return Vec3(-0x1p+0f, 0x1.777a5cp-25f, 0x0p+0f);
        case 7: return Vec3(0x1.6a09e6p-1f, 0x1.6a09e6p-1f, 0x0p+0f);
        case 8: return Vec3(-0x1.6a09e6p-1f, 0x1.6a09e6p-1f, 0x0p+0f);
        case 9: return Vec3(0x1.9bc4e4p-9f, 0x1.ffff5ap-1f, 0x0p+0f);
        default: return Vec3(-0x1.9bc4e4p-9f, 0x1.ffff5ap-1f, 0x0p+0f);
    }
}
CB_HDNI Vec3 force_preferred_vector(const Vec3 &src) {
    float best = -1.0f;
    Vec3 bv;
    for (int i = 0; i < 11; i++) {
        const Vec3 c = preferred_dir(i);
        float d = c.dot(src);
        if (d > best) {
            best = d;
            bv = c;
        }
    }
    return bv;
}
CB_HDNI float force_preferred_angle(float a) {
    float bestDiff = 10000.0;
    float bv = 0;
    for (int i = 0; i < 11; i++) {
        float d = fabsf(preferred_angle(i) - a);
        if (d < bestDiff) {
            bestDiff = d;
            bv = preferred_angle(i);
        }
    }
    return bv;
}
CB_HDNI float force_allowed_body_angle_value(float a) {
    const double f[5] = {0, 0.25, -0.25, 0.75, -0.75};
    float bestDiff = 10000.0;
    float bv = 0;
    for (int i = 0; i < 5; i++) {
        float c = (float)(f[i] * (double)kPi);
        float d = fabsf(c - a);
        if (d < bestDiff) {
            bestDiff = d;
            bv = c;
        }
    }
    return bv;
}
CB_HD float fast_cornering_bias(const Vec3 &cur, const Vec3 &des, float velExp, float bias) {
    float a = angle2d_to(des.normalized(cur), cur);
    float cmb = lm::lm_sinf(fabsf(a) - 0.5f * kPi) * 0.5f + 0.5f;
    float vb = lm::lm_powf(clampf_(cur.length() / (kSprintVel - 0.5f), 0.0f, 1.0f), velExp);
    return vb * cmb * bias;
}
CB_HD float stretch_sprint(const float &v, float inMax, float outMax) {
    if (v < kWalkSprintSwitch) return v;
    float part = v - kWalkSprintSwitch;
    float oldL = inMax - kWalkSprintSwitch, newL = outMax - kWalkSprintSwitch;
    float f = newL / oldL;
    return kWalkSprintSwitch + part * f;
}
CB_HD Vec3 front_of_foot_offset(float vel, float bodyAngleRel, float height) {
    float full = 1.0f;
    float dist = 0.34f + vel * kTouchOffset_ms * 0.001f * full;
    Vec3 fwd = Vec3(0, -dist * 0.8f, 0);
    float ba = bodyAngleRel;
    if (vel < kIdleDribbleSwitch) ba = 0;
    Vec3 ang = rot2d(Vec3(0, -dist * 0.2f, 0), ba);
    return (fwd + ang) * (1.0f - clampf_((height - 0.11f) / 4.0f, 0.0f, 0.5f));
}

// ---------------------------------------------------------------------------------------------
// Sorting. A chain of stable sorts by NaN-free `<` keys equals a sort of (key, position) pairs.
CB_HD bool pair_less(double ka, int ia, double kb, int ib) { return ka < kb || (!(kb < ka) && ia < ib); }

template <class KeyFn>
CB_HDNI void stable_sort(const Sim &s, AnimList &list, KeyFn key) {
    const int n = list.count;
    if (n < 2) return;
#if CB_DEVICE_PASS
    if (!crew_serial()) {
        // A crew sorts (key, position) pairs in the environment's scratch with a bitonic network.
        WarpScratch &sc = *s.scratch;
        int N = 1;
        while (N < n) N <<= 1;
        const int rank = crew_rank(), w = crew_width();
        crew_sync();
        {
            CrewDivided divided;
            for (int i = rank; i < N; i += w) {
                sc.keys[i] = i < n ? (double)key((int)list[i]) : (double)INFINITY;
                sc.idx[i] = (int16_t)(i < n ? i : 32767);
            }
        }
        crew_sync();
        for (int k = 2; k <= N; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                for (int t = rank; t < N / 2; t += w) {
                    // t-th pair of this stage: lower element i with bit j clear.
                    int i = ((t / j) * 2 * j) + (t % j);
                    int l = i + j;
                    bool up = (i & k) == 0;
                    double ki = sc.keys[i], kl = sc.keys[l];
                    int ii = sc.idx[i], il = sc.idx[l];
                    bool swap = up ? pair_less(kl, il, ki, ii) : pair_less(ki, ii, kl, il);
                    if (swap) {
                        sc.keys[i] = kl; sc.keys[l] = ki;
                        sc.idx[i] = (int16_t)il; sc.idx[l] = (int16_t)ii;
                    }
                }
                crew_sync();
            }
        }
        for (int i = rank; i < n; i += w) sc.list[i] = list[sc.idx[i]];
        crew_sync();
        for (int i = 0; i < n; i++) list[i] = sc.list[i];
        crew_sync();
        return;
    }
#endif
    if (crew_owns_env() && s.scratch) {
        // The lane owns the environment's scratch: each key once, then a bottom-up stable merge
        // sort of (key, position) runs, the left run winning ties.
        WarpScratch &sc = *s.scratch;
        double *ka = sc.keys, *kb = sc.keys2;
        int16_t *ia = sc.idx, *ib = sc.idx2;
        for (int i = 0; i < n; i++) {
            ka[i] = (double)key((int)list[i]);
            ia[i] = list[i];
        }
        for (int width = 1; width < n; width *= 2) {
            for (int lo = 0; lo < n; lo += 2 * width) {
                const int mid = lo + width < n ? lo + width : n;
                const int hi = lo + 2 * width < n ? lo + 2 * width : n;
                int l = lo, r = mid, o = lo;
                while (l < mid && r < hi) {
                    if (ka[r] < ka[l]) {
                        kb[o] = ka[r];
                        ib[o++] = ia[r++];
                    } else {
                        kb[o] = ka[l];
                        ib[o++] = ia[l++];
                    }
                }
                while (l < mid) {
                    kb[o] = ka[l];
                    ib[o++] = ia[l++];
                }
                while (r < hi) {
                    kb[o] = ka[r];
                    ib[o++] = ia[r++];
                }
            }
            double *kt = ka;
            ka = kb;
            kb = kt;
            int16_t *it = ia;
            ia = ib;
            ib = it;
        }
        for (int i = 0; i < n; i++) list[i] = ia[i];
        return;
    }
    // Serial stable insertion sort (nested inside a warp-shared environment).
    for (int i = 1; i < n; i++) {
        int16_t v = list[i];
        double kv = (double)key((int)v);
        int j = i - 1;
        while (j >= 0 && kv < (double)key((int)list[j])) {
            list[j + 1] = list[j];
            j--;
        }
        list[j + 1] = v;
    }
}

constexpr int kMaxChainKeys = 8;
CB_HD bool chain_precedes(const double *a, const double *b, int n) {
    for (int k = 0; k < n; k++) {
        if (a[k] < b[k]) return true;
        if (b[k] < a[k]) return false;
    }
    return false;
}
// The first element after a chain of stable sorts: the smallest keys in order (the last sort's
// key first), earliest position on a full tie.
template <class KeysFn>
CB_HDNI int first_of_chain(const AnimList &list, int nkeys, KeysFn keys) {
    const int n = list.count;
    if (n < 2) return list[0];
    const bool serial = crew_serial();
    const int rank = serial ? 0 : crew_rank(), w = serial ? 1 : crew_width();
    int best = -1;
    double bk[kMaxChainKeys];
    {
#if CB_DEVICE_PASS
        crew_sync();
        CrewDivided divided(!serial);
#endif
        for (int e = rank; e < n; e += w) {
            double ek[kMaxChainKeys];
            keys((int)list[e], ek);
            if (best < 0 || chain_precedes(ek, bk, nkeys)) {
                best = e;
                for (int k = 0; k < nkeys; k++) bk[k] = ek[k];
            }
        }
    }
#if CB_DEVICE_PASS
    if (!serial) {
        // Each lane holds the best of its share; a butterfly over the crew keeps the smallest keys,
        // the earliest position on a full tie, and every lane ends with the same answer.
        const unsigned mask = crew_mask();
        for (int off = w >> 1; off > 0; off >>= 1) {
            const int ob = __shfl_xor_sync(mask, best, off, w);
            double ok[kMaxChainKeys];
            for (int k = 0; k < nkeys; k++) ok[k] = __shfl_xor_sync(mask, bk[k], off, w);
            if (ob >= 0 && (best < 0 || chain_precedes(ok, bk, nkeys) ||
                            (!chain_precedes(bk, ok, nkeys) && ob < best))) {
                best = ob;
                for (int k = 0; k < nkeys; k++) bk[k] = ok[k];
            }
        }
    }
#endif
    return list[best];
}

// ---------------------------------------------------------------------------------------------
// Crude selection.
struct CrudeQuery {
    bool byFunctionType = false;
    int functionType = 0;
    bool heedForcedFoot = false;
    int strongFoot = 1;
    bool bySide = false;
    Vec3 lookAtVectorRelative;
    bool allowLastDitch = false;
    bool byIncomingVelocity = false, incomingVelocityStrict = false,
         incomingVelocityNoDribbleToIdle = false, incomingVelocityNoDribbleToSprint = false,
         incomingVelocityForceLinearity = false;
    int incomingVelocity = 0;
    bool byOutgoingVelocity = false;
    int outgoingVelocity = 0;
    bool byPickupBall = false, pickupBall = true;
    bool byIncomingBodyDirection = false;
    Vec3 incomingBodyDirection;
    bool incomingBodyDirectionStrict = false, incomingBodyDirectionForceLinearity = false;
    bool byIncomingBallDirection = false;
    Vec3 incomingBallDirection;
    bool byOutgoingBallDirection = false;
    Vec3 outgoingBallDirection;
    bool byTripType = false;
    int tripType = 0;
    int32_t incomingSpecialState = kSS_Empty, incomingRetainState = kSS_Empty;
    float specialVar1 = 0, specialVar2 = 0;
};

CB_HD bool check_function_type(int at, int ft) {
    switch (ft) {
        case kFtMovement: return at == kAS_Movement;
        case kFtBallControl: return at == kAS_BallControl;
        case kFtTrap: return at == kAS_Trap;
        case kFtShortPass: return at == kAS_ShortPass;
        case kFtLongPass: return at == kAS_LongPass;
        case kFtHighPass: return at == kAS_HighPass;
        case kFtShot: return at == kAS_Shot;
        case kFtDeflect: return at == kAS_Deflect;
        case kFtCatch: return at == kAS_Catch;
        case kFtInterfere: return at == kAS_Interfere;
        case kFtTrip: return at == kAS_Trip;
        case kFtSliding: return at == kAS_Sliding;
        case kFtSpecial: return at == kAS_Special;
        default: return false;
    }
}
// Bit-exact match of a direction against the allowed-direction table, -1 if none.
CB_HD int allowed_body_entry(const Vec3 &d) {
    for (int i = 0; i < 6; i++) {
        const Vec3 a = allowed_body_dir(i);
        if (f2u(d.c[0]) == f2u(a.c[0]) && f2u(d.c[1]) == f2u(a.c[1]) && f2u(d.c[2]) == f2u(a.c[2]))
            return i;
    }
    return -1;
}

CB_HDNI void crude_selection(const Sim &s, const CrudeQuery &q, AnimList &out) {
    out.count = 0;
    const AnimTables &T = s.T();
    const float margin = 0.06f * kPi;
    Vec3 fenced;
    float queryInToFence = 0.0f;
    if (q.bySide) {
        fenced = rot2d(q.lookAtVectorRelative, kPi);
        queryInToFence = angle2d_to(fenced, q.incomingBodyDirection);
    }
    const bool byBody = q.byIncomingBodyDirection && !(q.byIncomingVelocity && q.incomingVelocity == kVelIdle);
    const int qEntry = byBody ? allowed_body_entry(q.incomingBodyDirection) : -1;
    float qInBodyFixAbs = 0.0f, qIdleBodyAbs = 0.0f;
    if (byBody) {
        qInBodyFixAbs = fabsf(fix_angle(angle2d(q.incomingBodyDirection)));
        qIdleBodyAbs = fabsf(angle2d_to(Vec3(0, -1, 0), q.incomingBodyDirection));
    }
    const int16_t *lst = nullptr;
    int cand = T.animCount;
    if (q.byFunctionType && q.functionType >= 0 && q.functionType < kFunctionTypeSlots) {
        lst = T.functionAnims + T.functionOffsets[q.functionType];
        cand = T.functionOffsets[q.functionType + 1] - T.functionOffsets[q.functionType];
    }
    const bool qInBallNonzero = q.incomingBallDirection.length() != 0.0f;
    Vec3 qInBall = q.incomingBallDirection;
    qInBall.c[2] *= 0.4f;
    if (qInBallNonzero) qInBall.normalize();
    const Vec3 qOut2D = q.outgoingBallDirection.flat();
    const bool qOutNull = fabsf(qOut2D.c[0]) < 0.000001f && fabsf(qOut2D.c[1]) < 0.000001f &&
                          fabsf(qOut2D.c[2]) < 0.000001f;
    const Vec3 qOutN = qOutNull ? Vec3(0) : qOut2D.normalized(Vec3(0));
    auto pass = [&](int ai) -> bool {
        const Anim &a = T.anims[ai];
        const AnimDerived &d = T.derived[ai];
        int at = a.animationType;
        if (q.byFunctionType && !lst && !check_function_type(at, q.functionType)) return false;
        if (q.byIncomingVelocity) {
            int aiv = vel_category(a.incomingVelocity);
            if (!q.incomingVelocityStrict) {
                if (q.incomingVelocityNoDribbleToIdle && aiv == kVelIdle && q.incomingVelocity == kVelDribble) return false;
                if (aiv == kVelIdle && q.incomingVelocity == kVelWalk) return false;
                if (aiv == kVelIdle && q.incomingVelocity == kVelSprint) return false;
                if (aiv == kVelDribble && q.incomingVelocity == kVelIdle) return false;
                if (aiv == kVelWalk && q.incomingVelocity == kVelIdle) return false;
                if (aiv == kVelSprint && q.incomingVelocity == kVelIdle) return false;
                if (q.incomingVelocityNoDribbleToSprint && aiv == kVelSprint && q.incomingVelocity == kVelDribble)
                    return false;
                if (q.incomingVelocityForceLinearity) {
                    float ain = range_velocity(a.incomingVelocity);
                    float aout = range_velocity(a.outgoingVelocity);
                    float qin = vel_float(q.incomingVelocity);
                    if (vel_category(ain) == kVelDribble) ain = kWalkVel;
                    if (vel_category(aout) == kVelDribble) aout = kWalkVel;
                    if (vel_category(qin) == kVelDribble) qin = kWalkVel;
                    float upper = (qin < aout) ? aout : qin;
                    float lower = (aout < qin) ? aout : qin;
                    if (ain > upper) return false;
                    if (ain < lower) return false;
                }
            } else {
                if (aiv != q.incomingVelocity) return false;
            }
        }
        if (q.byOutgoingVelocity && vel_category(a.outgoingVelocity) != q.outgoingVelocity) return false;
        if (q.bySide) {
            const Vec3 &ain = a.incomingBodyDirection;
            const Vec3 &aout = d.crudeOutDirectionRotated;
            const float turn = d.crudeTurnAngle;
            if (fabsf(turn) > 0.06f * kPi) {
                int aside = (turn > 0) ? 0 : 1;
                float ainToFence = angle2d_to(fenced, ain);
                float fenceToOut = angle2d_to(aout, fenced);
                int ainToFenceSide = (ainToFence > 0) ? 0 : 1;
                int qInToFenceSide = (queryInToFence > 0) ? 0 : 1;
                int fenceToOutSide = (fenceToOut > 0) ? 0 : 1;
                if (ainToFenceSide == aside && fenceToOutSide == aside && fabsf(ainToFence + fenceToOut) < kPi)
                    return false;
                // GRF adds the side number (0/1) to an angle here; kept as written.
                if (qInToFenceSide == aside && fenceToOutSide == aside &&
                    fabsf((float)qInToFenceSide + fenceToOut) < kPi)
                    return false;
            }
        }
        if (q.byPickupBall) {
            if ((!d.outgoingRetainRaw && q.pickupBall) || (d.outgoingRetainRaw && !q.pickupBall)) return false;
        }
        if (!q.allowLastDitch && a.lastDitch) return false;
        if (byBody) {
            if (vel_category(a.incomingVelocity) != kVelIdle) {
                Vec3 ainBody = a.incomingBodyDirection;
                if (d.crudeInBodyFixAbsolute > qInBodyFixAbs + margin) return false;
                const Vec3 &aoutBody = d.crudeOutBodyDirection;
                const float qOffset = qEntry >= 0 ? d.incomingBodyAngles[qEntry]
                                                  : angle2d_to(ainBody, q.incomingBodyDirection);
                if (q.incomingBodyDirectionStrict) {
                    if (fabsf(qOffset) > margin) return false;
                } else {
                    if (fabsf(qOffset) > 0.5f * kPi + margin) return false;
                }
                if (q.incomingBodyDirectionForceLinearity) {
                    float bodyTurn = d.bodyTurnAngle;
                    (void)aoutBody;
                    if ((bodyTurn > margin && qOffset > margin) || (bodyTurn < -margin && qOffset < -margin))
                        return false;
                    if (fabsf(bodyTurn) + fabsf(qOffset) > kPi + margin) return false;
                }
            } else {
                if (q.incomingBodyDirectionStrict) {
                    if (qIdleBodyAbs > margin) return false;
                } else {
                    if (qIdleBodyAbs > 0.25f * kPi + margin) return false;
                }
            }
        }
        if (q.byIncomingBallDirection) {
            if (d.crudeInBallNonzero && qInBallNonzero) {
                float bda = fabsf(angle2d_to(qInBall, d.crudeInBallAdapted));
                float md = d.incomingMaxDeviation;
                if (md == 0.0f) {
                    md = T.maxIncomingBallDirDeviation.value();
                    if (at == kAS_Deflect) md = 0.4f * kPi;
                }
                if (bda > md) return false;
            }
        }
        if (q.byOutgoingBallDirection) {
            const Vec3 &abd = d.crudeBallDirectionNormalized;
            float bda = qOutNull && d.ballDirectionFinite
                            ? 0.0f
                            : fabsf(angle2d_to(qOutNull ? abd : qOutN, abd));
            float md = d.outgoingMaxDeviation;
            if ((double)md == 0.0) md = T.maxOutgoingBallDirDeviation.value();
            if (bda > md) return false;
        }
        if (q.incomingSpecialState != a.incomingSpecialState) return false;
        if ((q.functionType == kFtDeflect ||
             ((q.incomingRetainState != kSS_Empty) != (a.incomingRetainState != kSS_Empty))) &&
            q.incomingRetainState != a.incomingRetainState)
            return false;
        if (q.specialVar1 != a.specialVar1) return false;
        if (q.specialVar2 != a.specialVar2) return false;
        if (q.byTripType && d.tripTypeRounded != q.tripType) return false;
        if (q.heedForcedFoot && d.forcedFootWhich != 0) {
            int af = d.touchFootLeft ? 0 : 1;
            if (a.currentFoot == 0) af = af == 0 ? 1 : 0;
            if (d.forcedFootWhich == 1 && q.strongFoot != af) return false;
            if (d.forcedFootWhich == 2 && q.strongFoot == af) return false;
        }
        return true;
    };
    int count = 0;
    crew_filter(0, cand, [&](int c) { return pass(lst ? lst[c] : c); },
               [&](int c) { out[count++] = (int16_t)(lst ? lst[c] : c); });
    out.count = count;
}

struct Predicates {
    int desiredFoot = 0;
    int incomingVelocity = 0;
    Vec3 relDesiredDirection;
    float corneringBias = 0.0f;
    int desiredVelocity = 0;
    Vec3 relIncomingBodyDirection;
    Vec3 lookAt;  // world coordinates
    Vec3 relDesiredTripDirection;
    float idle = 0.0f;
};

CB_HD float movement_similarity(const Vec3 &outDir, const Vec3 &outMov, const Vec3 &relDesDir,
                                int desVel, float corneringBias) {
    Vec3 dm = relDesDir * vel_float(desVel);
    dm = dm * (1.0f - corneringBias);
    float v = (dm - outMov).length();
    v -= fabsf(relDesDir.dot(outDir)) * 4.0f;
    return v;
}
CB_HDNI float direction_similarity(const Anim &a, const Predicates &pr, const Vec3 &relLookAt) {
    Vec3 relBody = (relLookAt - a.translation).normalized(Vec3(0, -1, 0));
    float maxSmuggle = 0.1f * kPi;
    float outAngle = angle2d_to(
        rot2d(a.outgoingDirection, clampf_(angle2d_to(pr.relDesiredDirection, a.outgoingDirection),
                                           -maxSmuggle, maxSmuggle)),
        Vec3(0, -1, 0));
    Vec3 predBody = rot2d(a.outgoingBodyDirection, outAngle);
    float r = fabsf(angle2d_to(predBody, relBody));
    r += fabsf(a.outgoingBodyAngle.value()) * 0.05f;
    return r;
}
CB_HD float key_idle(const Anim &a, const Predicates &p) { return fabsf(a.idleLevel - p.idle); }
CB_HD int key_foot(const Anim &a, const Predicates &p) {
    int r = 1;
    if (a.currentFoot == p.desiredFoot) r = 0;
    if (vel_category(a.incomingVelocity) == kVelIdle) r = 0;
    return r;
}
CB_HD float key_incoming_velocity(const Anim &a, const Predicates &p) {
    int cur = velocity_id(p.incomingVelocity);
    int in = velocity_id(vel_category(a.incomingVelocity));
    float r = fabsf(clampf_((float)(in - cur), -3, 3));
    int out = velocity_id(vel_category(a.outgoingVelocity));
    int mx = cur > out ? cur : out, mn = cur < out ? cur : out;
    if (in > mx) r += 0.5f;
    if (in < mn) r += 0.5f;
    return r;
}
// |angle between allowed body directions i and j| / pi.
CB_HD float allowed_body_key(int i, int j) {
    const float t[36] = {0x0p+0f,   0x1p-2f, 0x1p-2f, 0x1.8p-1f, 0x1.8p-1f, 0x0p+0f,
                         0x1p-2f,   0x0p+0f, 0x1p-1f, 0x1p-1f,   0x1p+0f,   0x1p+0f,
                         0x1p-2f,   0x1p-1f, 0x0p+0f, 0x1p+0f,   0x1p-1f,   0x0p+0f,
                         0x1.8p-1f, 0x1p-1f, 0x1p+0f, 0x0p+0f,   0x1p-1f,   0x0p+0f,
                         0x1.8p-1f, 0x1p+0f, 0x1p-1f, 0x1p-1f,   0x0p+0f,   0x0p+0f,
                         0x0p+0f,   0x1p+0f, 0x0p+0f, 0x0p+0f,   0x0p+0f,   0x0p+0f};
    return t[6 * i + j];
}
CB_HDNI float closest_opponent_distance(const Sim &s, int p) {
    const Match &w = s.w;
    const int opp = 1 - w.playerTeamID[p];
    const Vec3 pos = hum(w, p).spatial.position;
    float cd = 10000;
    int closest = -1;
    for (int o = 0; o < w.m.playerCount; o++) {
        if (w.playerTeamID[o] != opp || !w.m.players[o].base.isActive) continue;
        float d = (hum(w, o).spatial.position - pos).length();
        if (d < cd) {
            cd = d;
            closest = o;
        }
    }
    if (closest < 0) {
        s.fail(kStatusUnsupported);
        return 0.0f;
    }
    return get_distance(hum(w, closest).spatial.position, pos);
}
// curve(nclamp(10*frame, 0, 160)) for frames 0..16.
CB_HD float physics_curved_time(int frame) {
    const float t[17] = {0x0p+0f, 0x1.3ad04p-7f, 0x1.37ca2p-5f, 0x1.59267p-4f, 0x1.2bec34p-3f,
                         0x1.c71898p-3f, 0x1.3c10eap-2f, 0x1.9c1d2p-2f, 0x1p-1f, 0x1.31f17p-1f,
                         0x1.61f78cp-1f, 0x1.8e39dap-1f, 0x1.b504f4p-1f, 0x1.d4db32p-1f,
                         0x1.ec835ep-1f, 0x1.fb14cp-1f, 0x1p+0f};
    return t[frame < 0 ? 0 : frame > 16 ? 16 : frame];
}
CB_HD float line_closest_to_point(const Vec3 &a, const Vec3 &b, const Vec3 &p) {
    if (a == b) return 0.0f;
    float ld = (b - a).length();
    if (ld < 0.000001f) return 0.0f;
    return ((p.c[0] - a.c[0]) * (b.c[0] - a.c[0]) + (p.c[1] - a.c[1]) * (b.c[1] - a.c[1])) / (ld * ld);
}
CB_HDNI int string_to_function_type(int at) {
    switch (at) {
        case kAS_Movement: return kFtMovement;
        case kAS_BallControl: return kFtBallControl;
        case kAS_Trap: return kFtTrap;
        case kAS_ShortPass: return kFtShortPass;
        case kAS_LongPass: return kFtLongPass;
        case kAS_HighPass: return kFtHighPass;
        case kAS_Shot: return kFtShot;
        case kAS_Deflect: return kFtDeflect;
        case kAS_Catch: return kFtCatch;
        case kAS_Interfere: return kFtInterfere;
        case kAS_Trip: return kFtTrip;
        case kAS_Sliding: return kFtSliding;
        case kAS_Special: return kFtSpecial;
    }
    return kFtNone;
}
CB_HD Vec3 outgoing_movement_of(const PosList &p) {
    if (p.count < 2) return Vec3(0);
    return (p[p.count - 1] - p[p.count - 2]) * 100.0f;
}

struct Selector {
    const Sim &s;
    int hi;  // humanoid index: players, then officials
    Predicates pr;
    struct TurnCache {
        bool valid = false;
        uint32_t bits = 0;
        lm::SinCosF t{0.0f, 1.0f};
    } fwdTurn, backTurn;

    CB_HD Selector(const Sim &sim, int humanoidIndex) : s(sim), hi(humanoidIndex) {}

    CB_HD static lm::SinCosF cached(TurnCache &c, float angle, float arg) {
        const uint32_t b = f2u(angle);
        if (!c.valid || c.bits != b) {
            c.t = lm::lm_sincosf(arg);
            c.bits = b;
            c.valid = true;
        }
        return c.t;
    }
    CB_HD lm::SinCosF turn(float a) { return cached(fwdTurn, a, a); }
    // Computed apart from `turn`: lm_cosf is not shown to be even.
    CB_HD lm::SinCosF back(float a) { return cached(backTurn, a, -a); }
    CB_HD static Vec3 rotby(const Vec3 &v, const lm::SinCosF &t) { return rot2d_cs(v, t.c, t.s); }

    CB_HD Match &w() const { return s.w; }
    CB_HD bool official() const { return hi >= s.w.m.playerCount; }
    CB_HD Player &player() const { return s.w.m.players[hi]; }
    CB_HD Humanoid &H() const { return any_hum(s.w, hi); }
    CB_HD SpatialState &SP() const { return H().spatial; }
    CB_HD const Anim &A(int i) const { return s.A(i); }
    CB_HD const AnimDerived &D(int i) const { return s.D(i); }

    CB_HD Vec3 rel_look_at() { return rotby(pr.lookAt - SP().position, back(SP().angle.value())); }
    CB_HD float movement_similarity_key(int i) {
        const AnimDerived &d = D(i);
        return movement_similarity(d.preferredOutgoingDirection, d.preferredOutgoingMovement,
                                   pr.relDesiredDirection, pr.desiredVelocity, pr.corneringBias);
    }
    CB_HD int incoming_body_query() { return force_allowed_body_index(pr.relIncomingBodyDirection); }
    CB_HD float incoming_body_key(int i, int qi) {
        float r = allowed_body_key(D(i).incomingBodyIndex, qi);
        if (vel_category(A(i).incomingVelocity) == kVelIdle) r = 0;
        return r;
    }
    CB_HD float preferred_out_angle(int i) { return D(i).preferredOutgoingAngle; }
    CB_HD float look_angle(int i) { return D(i).lookAngle; }
    CB_HD Vec3 smoothed_movement(int i, uint32_t frame) {
        const Anim &a = A(i);
        const int32_t off = D(i).smoothedMovementOffset;
        if (off >= 0 && frame < (uint32_t)a.positionCount) return s.T().smoothed[off + frame];
        return movement_at_frame(s.T().positions + a.firstPosition, a.positionCount, frame, 1);
    }
    CB_HD int mental_image() { return mental_index(s.w, H().mentalImageTime); }
    CB_HD Vec3 mental_ball_at(int t) { return mental_ball(s.w, mental_image(), t); }
    CB_HD float stat(int st) {
        return official() ? s.ctx.staticData->data[hi].statistics[st] : statistic(s, hi, st);
    }
    CB_HD float base_last_touch_bias(int decay) {
        uint64_t last = official() ? s.w.m.officials[hi - s.w.m.playerCount].lastTouchTime_ms
                                   : player().base.lastTouchTime_ms;
        if (decay > 0)
            return 1.0f - clampf_((float)(s.w.m.actualTime_ms - last) / (float)decay, 0.0f, 1.0f);
        return 0.0f;
    }
    CB_HD void set_movement_predicate(const Vec3 &relDes, int desVel) {
        pr.relDesiredDirection = relDes;
        pr.desiredVelocity = desVel;
        pr.corneringBias = fast_cornering_bias(Vec3(0, -1.0f * SP().floatVelocity, 0),
                                               relDes * vel_float(desVel), 1.0f, 0.9f);
    }
    template <class F>
    CB_HD void sort(AnimList &l, F key) { stable_sort(s, l, key); }
    CB_HD void sort_base(AnimList &l) {
        sort(l, [&](int i) { return A(i).baseAnimation ? 0 : 1; });
    }
    CB_HD void sort_incoming_body(AnimList &l) {
        const int qi = l.count > 1 ? incoming_body_query() : 0;
        sort(l, [&](int i) { return incoming_body_key(i, qi); });
    }
    CB_HD bool allow_last_ditch(bool withPossession = true) {
        if (withPossession && team_of(s.w, hi).teamPossessionAmount < 1.0f) return true;
        return ((int)player().timeNeededToGetToBallOptimistic_ms * 1.7f + 800 <
                (float)(int)player().timeNeededToGetToBall_ms);
    }
    CB_HD bool high_or_bouncy() {
        const Ball &b = s.w.m.ball;
        float h1 = ball_predict(b, 10).c[2];
        float h2 = ball_predict(b, kTouchOffset_ms).c[2];
        float bounce = fabsf(b.momentum.c[2]);
        if (h1 > 0.3f || h2 > 0.3f) return true;
        if (bounce > 1.0f) return true;
        return false;
    }

    CB_HDNI void keep_best_direction(AnimList &l, const PlayerCommand &cmd, bool strict,
                                     float allowedAngle = 0, int allowedVelSteps = 0, int forcedQuadrant = -1) {
        const AnimTables &T = s.T();
        int bestQ = forcedQuadrant;
        if (bestQ == -1) {
            sort(l, [&](int i) { return movement_similarity_key(i); });
            if (strict && cmd.desiredFunctionType != kFtMovement) sort_base(l);
            bestQ = A(l[0]).quadrantID;
        }
        int kept = 1;
        crew_filter(1, l.count,
                   [&](int c) {
                       const Anim &a = A(l[c]);
                       if (strict) return a.quadrantID == bestQ;
                       const Quadrant &bq = T.quadrants[bestQ];
                       const Quadrant &qq = T.quadrants[a.quadrantID];
                       bool ok = true;
                       if (!a.lastDitch) {
                           int dv = velocity_id(qq.velocity, true) - velocity_id(bq.velocity, true);
                           if ((dv < 0 ? -dv : dv) > allowedVelSteps) ok = false;
                       }
                       if (fabsf(qq.angle.value() - bq.angle.value()) > allowedAngle) ok = false;
                       return ok;
                   },
                   [&](int c) { l[kept++] = l[c]; });
        l.count = kept;
    }
    CB_HDNI void keep_best_body_direction(AnimList &l, const PlayerCommand &cmd, bool strict,
                                          float allowedAngle = 0) {
        Vec3 rla;
        if (l.count > 1) rla = rel_look_at();
        sort(l, [&](int i) { return direction_similarity(A(i), pr, rla); });
        if (strict && cmd.desiredFunctionType != kFtMovement) sort_base(l);
        float bestLook = look_angle(l[0]);
        int kept = 1;
        crew_filter(1, l.count,
                   [&](int c) {
                       float la = look_angle(l[c]);
                       float aa = 0.06f * kPi;
                       if (!strict) aa = allowedAngle;
                       return fabsf(la - bestLook) <= aa;
                   },
                   [&](int c) { l[kept++] = l[c]; });
        l.count = kept;
    }

    CB_HDNI int idle_movement_animation() {
        CrudeQuery q;
        q.byFunctionType = true;
        q.functionType = kFtMovement;
        q.byIncomingVelocity = true;
        q.incomingVelocity = kVelIdle;
        q.byOutgoingVelocity = true;
        q.outgoingVelocity = kVelIdle;
        AnimList l;
        crude_selection(s, q, l);
        pr.idle = 1;
        pr.relIncomingBodyDirection = Vec3(0, -1, 0);
        pr.incomingVelocity = kVelIdle;
        set_movement_predicate(Vec3(0, -1, 0), kVelIdle);
        pr.lookAt = SP().position + rotby(Vec3(0, -10, 0), turn(SP().angle.value()));
        Vec3 rla;
        int qi = 0;
        if (l.count > 1) {
            rla = rel_look_at();
            qi = incoming_body_query();
        }
        if (l.count == 0) {
            s.fail(kStatusUnsupported);
            return 0;
        }
        return first_of_chain(l, 5, [&](int i, double *k) {
            k[0] = movement_similarity_key(i);
            k[1] = direction_similarity(A(i), pr, rla);
            k[2] = key_incoming_velocity(A(i), pr);
            k[3] = incoming_body_key(i, qi);
            k[4] = key_idle(A(i), pr);
        });
    }

    struct PhysicsFrame {
        Vec3 animMovement, adaptedAnimMovement, normalizedMax, normalizedAdapted;
        float adaptedAnimVelocity, rotCos, rotSin, curvedTime;
    };

    // The positions (start-relative) an animation produces with the player's physics, and the
    // outgoing movement; `rotOffset` receives the rotation smuggle.
    CB_HDNI Vec3 physics_vector(int ai, bool useDesMov, const Vec3 &desMov, bool useDesBody,
                                const Vec3 &desBodyRel, PosList &out, float &rotOffset) {
        (void)useDesBody;
        const Anim &a = A(ai);
        const AnimDerived &d = D(ai);
        SpatialState &sp = SP();
        const float angle = sp.angle.value();
        const lm::SinCosF t = turn(angle);
        out.count = 0;
        int touchFrame = d.touchFrame;
        bool touch = (touchFrame > 0);
        float stAgility = stat(kStPhysicalAgility);
        float stAccel = stat(kStPhysicalAcceleration);
        float stDribble = stat(kStTechnicalDribble);
        float inSwitch = 0.0f, outSwitch = 0.0f;
        const int at = a.animationType;
        if (at == kAS_BallControl) outSwitch = 0.0f;
        else if (at == kAS_Trap) outSwitch = 0.0f;
        else if (at == kAS_Interfere) outSwitch = 0.0f;
        else if (at == kAS_Deflect) outSwitch = 1.0f;
        else if (at == kAS_Sliding) outSwitch = 0.0f;
        else if (at == kAS_Special) outSwitch = 1.0f;
        else if (at == kAS_Trip) outSwitch = 0.5f;
        else if (touch) outSwitch = 1.0f;
        if (a.incomingSpecialState != kSS_Empty || a.outgoingSpecialState != kSS_Empty) outSwitch = 1.0f;
        Vec3 animIn = rotby(Vec3(0, -1, 0), t) * range_velocity(a.incomingVelocity);
        Vec3 adCur = animIn * inSwitch + sp.movement * (1.0f - inSwitch);
        Vec3 predOut = rotby(a.outgoingMovement, t);
        Vec3 velDes = useDesMov ? desMov : predOut;
        Vec3 adDes = predOut * outSwitch + velDes * (1.0f - outSwitch);
        const float playerMax = max_velocity(*s.ctx.staticData, hi);
        float maxVel = playerMax;
        if (touch) maxVel *= 0.92f;
        const int dt = 10;
        float diff = d.animDifficultyFactor;
        float diffPenalty = lm::lm_powf_pos(
            clampf_((diff - 0.0f) * (1.0f - (stAgility * 0.2f + stAccel * 0.2f)) * 2.0f, 0.0f, 1.0f), 0.7f);
        float powerF = 1.0f - clampf_(lm::lm_powf_pos(base_last_touch_bias(1000), 0.8f) * (0.8f - stDribble * 0.3f),
                                      0.0f, 0.4f);
        powerF *= 1.0f - clampf_(H().decayingPositionOffset.length() * (10.0f - stat(kStPhysicalBalance) * 5.0f) - 0.1f,
                                 0.0f, 0.3f);
        Vec3 temporal = adCur;
        Vec3 curPos;
        float physicsBias = 1.0f;
        float maUnder = 0.125f * kPi, maOver = 0.125f * kPi, maStraight = 0.125f * kPi;
        if (touch) {
            float bonus = 1.0f - lm::lm_powf_pos(nclamp((adCur + predOut).length() * 0.5f, 0, kSprintVel), 0.8f) * 0.8f;
            bonus *= 0.6f + 0.4f * stat(kStTechnicalBallControl);
            maUnder = 0.2f * kPi * bonus;
            maOver = 0;
            maStraight = 0.1f * kPi * bonus;
        }
        if (at == kAS_Sliding) {
            maUnder = 0.5f * kPi;
            maOver = 0.5f * kPi;
            maStraight = 0.5f * kPi;
        }
        if (at == kAS_Movement) physicsBias *= 1.0f;
        if (at == kAS_BallControl) physicsBias *= 1.0f;
        if (at == kAS_Trap) physicsBias *= 1.0f;
        if (at == kAS_ShortPass) physicsBias *= 0.0f;
        if (at == kAS_HighPass) physicsBias *= 0.0f;
        if (at == kAS_Shot) physicsBias *= 0.0f;
        if (at == kAS_Interfere) physicsBias *= 0.5f;
        if (at == kAS_Deflect) physicsBias *= 0.0f;
        if (at == kAS_Sliding) physicsBias *= 1.0f;
        if (at == kAS_Trip) {
            if (d.tripTypeIsOne) physicsBias *= 0.5f;
            else physicsBias *= 0.0f;
        }
        if (at == kAS_Special) physicsBias *= 0.0f;
        if (a.incomingSpecialState != kSS_Empty) physicsBias *= 0.0f;
        const float accelMul = 0.5f + 0.5f;
        float capped = 0;
        if (physicsBias > 0.0f) {
            Vec3 aov = predOut.normalized(Vec3(0));
            if (vel_category(predOut.length()) == kVelIdle) aov = rotby(a.outgoingDirection, t);
            Vec3 dv = adDes.normalized(Vec3(0));
            if (vel_category(adDes.length()) == kVelIdle) dv = rotby(desBodyRel, t);
            float toDes = angle2d_to(dv, aov);
            if (fabsf(toDes) <= 0.5f * kPi || at == kAS_Sliding) {
                float change = angle2d_to(aov, sp.directionVector);
                if (fabsf(change) > 0.06f * kPi) {
                    int sg = sign_side(change);
                    if (sign_side(toDes) == sg) capped = clampf_(toDes, -maOver, maOver);
                    else capped = clampf_(toDes, -maUnder, maUnder);
                } else {
                    capped = clampf_(toDes, -maStraight, maStraight);
                }
            }
        }
        const int effFrames = a.frameCount - 1;
        const float adDesVel = adDes.length();
        const Vec3 adDesDir = adDes.normalized(Vec3(0));
        auto pre = [&](int frame) {
            const int tms = frame * dt;
            float fb = (tms + 10) / (float)((effFrames + 1) * 10);
            float lag = 1.0f;
            if (physicsBias > 0.0f && (at == kAS_BallControl || at == kAS_Movement)) {
                lag = 1.4f - 0.5f * 0.8f;
                lag *= 1.2f - stAgility * 0.4f;
                if (touch) lag += -0.1f + clampf_(diff * 0.4f, 0.0f, 0.5f);
                else lag += -0.2f + clampf_(diff * 0.2f, 0.0f, 0.2f);
                lag = clampf_(lag, 0.25f, 4.0f);
                if (touch && tms < touchFrame * 10) lag = std_max(lag, 0.7f);
                lag = lag * physicsBias + 1.0f * (1.0f - physicsBias);
            }
            float afb = lag == 1.0f ? fb : lm::lm_powf(fb, lag);
            Vec3 am = rotby(smoothed_movement(ai, cvt_f_u32(effFrames * afb)), t);
            float av = am.length();
            Vec3 aam = am;
            float aav = av;
            if (av > kWalkSprintSwitch && (at == kAS_Movement || at == kAS_BallControl || at == kAS_Trap)) {
                if (maxVel > av) {
                    aav = stretch_sprint(av, kAnimSprintVel, maxVel);
                    aam = aam.normalized(Vec3(0)) * aav;
                }
            }
            PhysicsFrame f;
            f.animMovement = am;
            f.adaptedAnimMovement = aam;
            f.adaptedAnimVelocity = aav;
            f.normalizedMax = normalized_max(aam, 1.0f);
            f.normalizedAdapted = aam.normalized(Vec3(0));
            const float rot = capped * fb;
            // Below 2^-12 the sine is the argument and the cosine 1 (the tests of sinf / cosf).
            if (lm::top12f(rot) < lm::top12f(0x1p-12f)) {
                f.rotCos = 1.0f;
                f.rotSin = rot;
            } else {
                const lm::SinCosF ft = lm::lm_sincosf(rot);
                f.rotCos = ft.c;
                f.rotSin = ft.s;
            }
            f.curvedTime = physics_curved_time(frame);
            return f;
        };
        crew_pipeline<PhysicsFrame>(a.frameCount, pre, [&](int frame, const PhysicsFrame &f) {
            const int tms = frame * dt;
            float fb = (tms + 10) / (float)((effFrames + 1) * 10);
            const Vec3 &am = f.animMovement;
            Vec3 aam = f.adaptedAnimMovement;
            float aav = f.adaptedAnimVelocity;
            float maxSlower = 1.6f;
            if (touch) maxSlower = 1.2f;
            float maxFaster = 0.0f;
            const float tl = temporal.length();
            if (tl > aav) maxFaster = std_min(0.0f + 1.0f * (1.0f - fb), std_max(maxFaster, tl - aav));
            if (maxFaster > 0) maxFaster *= std_max(0.0f, f.normalizedMax.dot(adDesDir));
            if (at == kAS_Sliding) maxFaster = 100;
            const float desVel = adDesVel;
            aav = clampf_(desVel, aav - maxSlower, aav + maxFaster);
            aam = f.normalizedAdapted * aav;
            Vec3 res = aam;
            res = rot2d_cs(res, f.rotCos, f.rotSin);
            res = res * physicsBias + am * (1.0f - physicsBias);
            Vec3 toDes = (res - temporal);
            float brake = 0.0f;
            {
                Vec3 pm = temporal + toDes;
                float startVel = kIdleDribbleSwitch;
                if (tl > startVel && pm.length() > startVel) {
                    const Vec3 pd = pm.normalized(), td = temporal.normalized();
                    float maf = 1.0f * (dt / 1000.0f);
                    maf *= (0.7f + 0.3f * stAgility);
                    if (!touch) maf *= 1.5f;
                    float maxAngle = maf * kPi;
                    float vf = nclamp(tl, 0, kSprintVel);
                    maxAngle = maxAngle / (vf + 0.01f);
                    float ca = angle2d_to(pd, td);
                    if (fabsf(ca) > maxAngle) {
                        float over = fabsf(ca) - maxAngle;
                        toDes += -temporal * clampf_(over / kPi * 3.0f, 0.0f, 1.0f);
                    }
                }
            }
            {
                float maxChange = 0.03f;
                if (at == kAS_Trip) maxChange *= 0.7f;
                if (at == kAS_Sliding) maxChange = 0.1f;
                float vf = lm::lm_powf_pos(nclamp(tl, 0, kSprintVel), 1.5f);
                float fsf = vf;
                if (at == kAS_Movement) fsf *= 0.4f;
                maxChange *= (1.0f - fsf) + fsf * f.curvedTime;
                maxChange *= 1.2f - vf * 0.4f;
                maxChange *= 0.75f + 0.5f * 0.5f;
                maxChange *= powerF;
                float dl = toDes.length();
                float maxAdd = maxChange * dt;
                normalize_max(toDes, std_min(dl, maxAdd));
            }
            if (at != kAS_Sliding && at != kAS_Deflect) {
                float velExp = 1.8f;
                float accelPower = 11.0f * accelMul;
                float falloff = kIdleDribbleSwitch;
                const float nl = (temporal + toDes).length();
                if (nl > falloff) {
                    accelPower *= 1.0f - diffPenalty * 0.4f;
                    float air = clampf_(
                        lm::lm_powf_pos(clampf_((tl - falloff) / (playerMax - falloff), 0.0f, 1.0f), velExp),
                        0.0f, 1.0f);
                    Vec3 fwd;
                    if (nl > tl) {
                        Vec3 dest = temporal + toDes;
                        float v = tl;
                        float acc = nl - v;
                        fwd = dest.normalized(Vec3(0)) * acc;
                    }
                    float accAdd = fwd.length();
                    float maxAccPerSec = accelPower * (1.0f - air) * (stAccel * 0.3f + 0.7f);
                    float maxAccAdd = maxAccPerSec * (dt / 1000.0f);
                    if (accAdd > maxAccAdd) {
                        float rem = maxAccAdd / accAdd;
                        toDes = toDes - fwd * (1.0f - rem);
                    }
                }
            }
            Vec3 tt = temporal + toDes;
            if (tms >= (a.frameCount - 2) * 10) {
                if (vel_category(a.outgoingVelocity) == kVelIdle && vel_category(tt.length()) != kVelIdle)
                    tt = Vec3(0);
                else if (vel_category(a.outgoingVelocity) != kVelIdle && vel_category(tt.length()) == kVelIdle)
                    tt = normalized_to(rotby(a.outgoingMovement, t), kDribbleVel);
            }
            temporal = tt;
            if (tms >= (a.frameCount - 2) * 10) brake = 0.0f;
            curPos += temporal * (1.0f - brake) * (dt / 1000.0f);
            out[frame] = curPos;
        });
        out.count = a.frameCount > 0 ? a.frameCount : 0;
        Vec3 resMov = temporal;
        if (vel_category(a.outgoingVelocity) != kVelIdle && vel_category(resMov.length()) != kVelIdle)
            rotOffset = angle2d_to(rotby(resMov, back(angle)), a.outgoingMovement);
        else
            rotOffset = capped * physicsBias;
        return resMov;
    }

    CB_HDNI bool need_touch(int ai, const PlayerCommand &cmd) {
        const Anim &a = A(ai);
        SpatialState &sp = SP();
        // Never true (a bool as float is idle) but kept as written.
        if (vel_category((float)(a.outgoingVelocity != (float)kVelIdle)) != kVelIdle) return true;
        if (cmd.desiredVelocityFloat > kIdleDribbleSwitch) return true;
        if (fabsf(s.w.m.ball.momentum.length()) > 2.0f) return true;
        Vec3 am = rotby(a.outgoingMovement, turn(sp.angle.value())) * 0.3f + sp.movement * 0.7f;
        float av = am.length();
        am.normalize(sp.directionVector);
        am *= sp.movement.length() * 0.8f + av * 0.2f;
        Vec3 bm = (mental_ball_at(250).flat() - mental_ball_at(240).flat()) * 100;
        if (fabsf(a.outgoingAngle.value()) > 0.125f * kPi) return true;
        float dd = (am - bm).length();
        if ((double)dd >= 2.0) return true;
        float vd = am.length() - bm.length();
        if ((double)vd < -1.4 || (double)vd >= 0.7) return true;
        if (vel_category(a.outgoingVelocity) != kVelIdle) {
            float ad = am.normalized(sp.directionVector).dot(bm.normalized(sp.directionVector));
            if ((double)ad < 0.975) return true;
        }
        return false;
    }

    CB_HDNI void predicted_situation(Vec3 &pos, float &ang) {
        AnimationState &ca = H().anim;
        const Anim &a = A(ca.anim);
        SpatialState &sp = SP();
        if ((uint32_t)ca.positions.count > (uint32_t)ca.frameNumber) {
            pos = sp.position + ca.positions[a.frameCount - 1] + ca.actionSmuggle + ca.actionSmuggleSustain +
                  ca.movementSmuggle;
        } else {
            pos = sp.position + rot2d(a.translation.flat(), sp.angle.value()) + ca.actionSmuggle +
                  ca.actionSmuggleSustain + ca.movementSmuggle;
        }
        ang = sp.angle.value() + a.outgoingAngle.value() + ca.rotationSmuggle.end.value();
        ang = wrap_range(-kPi, kPi, ang);
    }
    CB_HD int desired_time_to_ball_ms() {
        return cvt_f_i32(clampf_((float)player().desiredTimeToBall_ms, (float)(int)player().timeNeededToGetToBall_ms,
                                 1000000.0f));
    }
    CB_HDNI Vec3 movement_smuggle() {
        AnimationState &ca = H().anim;
        const Anim &a = A(ca.anim);
        const MatchState &m = s.w.m;
        if (team_of(s.w, hi).designatedTeamPossessionPlayer != hi || m.designatedPossessionPlayer != hi ||
            ca.touchFrame != -1 || (ca.functionType == kFtTrip && !D(ca.anim).tripTypeIsOne) ||
            a.incomingSpecialState != kSS_Empty || a.outgoingSpecialState != kSS_Empty || !m.inPlay ||
            m.inSetPiece || m.ballRetainer != -1)
            return Vec3(0);
        Vec3 toDes;
        uint32_t ttb = (uint32_t)(int)player().timeNeededToGetToBall_ms;
        if (desired_time_to_ball_ms() > (int)ttb) ttb = (uint32_t)desired_time_to_ball_ms();
        uint32_t animTime = (uint32_t)a.frameCount * 10;
        uint32_t fut = animTime + kTouchOffset_ms > ttb ? animTime + kTouchOffset_ms : ttb;
        Vec3 predOut;
        if (ca.positions.count >= 2)
            predOut = (ca.positions[ca.positions.count - 1] - ca.positions[ca.positions.count - 2]) * 100.0f;
        Vec3 predPos;
        float predAng;
        predicted_situation(predPos, predAng);
        Vec3 bp = mental_ball_at((int)fut);
        float bh = bp.c[2];
        Vec3 foot = rot2d(front_of_foot_offset(predOut.length(), a.outgoingBodyAngle.value(), bh), predAng);
        Vec3 desBall = predPos + foot;
        if (!player().hasPossession) {
            Vec3 bs = mental_ball_at(0).flat();
            Vec3 be = mental_ball_at((int)fut).flat();
            if ((bs - be).length() < 0.5f) return Vec3(0);
            float frac = 0.0f;
            if (!(bs == be)) {
                float ld = (be - bs).length();
                if (!(ld < 0.000001f))
                    frac = ((desBall.c[0] - bs.c[0]) * (be.c[0] - bs.c[0]) + (desBall.c[1] - bs.c[1]) * (be.c[1] - bs.c[1])) /
                           (ld * ld);
            }
            Vec3 closest = bs + (be - bs) * frac;
            toDes = closest - desBall;
        } else {
            toDes = bp.flat() - desBall;
        }
        uint32_t maxEffect = 250 + kTouchOffset_ms;
        if (vel_category(a.outgoingVelocity) == kVelIdle) maxEffect = 2000;
        float maxEffectVel = kDribbleWalkSwitch;
        float maxSmugglePerSec = 1.6f;
        if (fut - (animTime + kTouchOffset_ms) > maxEffect) return Vec3(0);
        Vec3 toDesMov = toDes / (animTime * 0.001f);
        Vec3 resMov = predOut + toDesMov;
        float pv = predOut.length(), rv = resMov.length();
        if (rv > pv && rv > maxEffectVel) return Vec3(0);
        normalize_max(toDes, maxSmugglePerSec * ((a.frameCount - 1) * 0.01f));
        float removeDist = 0.06f;
        toDes = toDes.normalized(Vec3(0)) * std_max(0.0f, toDes.length() - removeDist);
        return toDes;
    }
    CB_HD float last_touch_bias_at(int decay, uint64_t t) {
        uint64_t at = t;
        if (t == 0) at = s.w.m.actualTime_ms;
        if (decay > 0)
            return 1.0f - clampf_((float)(at - player().base.lastTouchTime_ms) / (float)decay, 0.0f, 1.0f);
        return 0.0f;
    }

    CB_HDNI static float body_ball_advantage(const Anim &a, const Vec3 &touchMov, const Vec3 &inMov,
                                             const Vec3 &outMov, float outAngle, const Vec3 &bodyPos,
                                             const Vec3 &foot, const Vec3 &animBall2D,
                                             const Vec3 &actualBall2D, float radiusFactor,
                                             float radiusCheat) {
        const float cheatFactor = 0.5f, cheatBonus = 0.02f;
        float inV = inMov.length();
        float outV = outMov.length();
        float avgV = (inMov + outMov).length() * 0.5f;
        float vChange = outV - inV;
        float vChangePerSec = vChange / (a.frameCount * 0.01f);
        (void)touchMov;
        float bab = 1.0f - curve(nclamp(((bodyPos + foot.normalized(Vec3(0)) * 0.1f) - animBall2D).length(), 0.0f, 0.7f), 0.7f);
        float bacb = 1.0f - curve(nclamp(((bodyPos + foot.normalized(Vec3(0)) * 0.1f) - actualBall2D).length(), 0.0f, 0.7f), 0.4f);
        float vb = 1.0f - nclamp(avgV, kIdleVel, kSprintVel);
        float vcb = 1.0f - nclamp(vChangePerSec / 20.0f, -1.0f, 1.0f);
        float radius = radiusFactor;
        radius *= 1.0f + 1.0f * bab + 0.6f * bacb + 0.8f * bab * bacb + 0.0f * vcb + 1.0f * vb;
        float erc = radiusCheat;
        Vec3 outDir;
        if (vel_category(outMov.length()) == kVelIdle) outDir = rot2d(Vec3(0, -1, 0), outAngle);
        else outDir = outMov.normalized();
        Vec3 behindU = -(inMov * 0.1f + touchMov * 0.2f + outMov * 0.7f);
        Vec3 behind = behindU.normalized(Vec3(0)) * lm::lm_powf_pos(nclamp(behindU.length(), 0, kSprintVel), 0.5f);
        float dot = Vec3(0, -1, 0).dot(outDir);
        dot = 0.5f + clampf_(dot * 0.5f + 0.5f, 0.0f, 1.0f) * 0.5f;
        behind *= dot;
        Vec3 a2a = actualBall2D - animBall2D;
        {
            Vec3 sau = inMov;
            Vec3 sa = sau.normalized(outDir);
            float toStraight = angle2d_to(Vec3(0, -1, 0), sa);
            rot2d_inplace(a2a, toStraight);
            float lrf = 0.6f - 0.3f * lm::lm_powf_pos(nclamp(sau.length(), kIdleVel, kSprintVel), 0.7f);
            a2a.c[0] /= lrf;
            radius *= lm::lm_powf(1.0f / lrf, 0.5f);
            rot2d_inplace(a2a, -toStraight);
        }
        Vec3 adActual = animBall2D + a2a;
        float behindBias = 0.6f;
        Vec3 behindCenter = animBall2D + behind * (radius + (erc * behindBias)) * cheatFactor;
        float result = 1.0f;
        float allowed = (radius + erc) * cheatFactor + cheatBonus;
        if (get_distance(adActual, behindCenter) > allowed) result = 0.0f;
        return result;
    }

    CB_HDNI int best_cheatable(const AnimList &sorted, bool useDesMov, const Vec3 &desDir, float desVel,
                               bool useDesBody, const Vec3 &desBodyRel, PosList &posOut, int &touchFrameOut,
                               Vec3 &touchPosOut, Vec3 &smuggleOut, float &rotSmuggleOut,
                               bool preferPassAndShot = false) {
        const MatchState &m = s.w.m;
        SpatialState &sp = SP();
        const float angle = sp.angle.value();
        const bool retainerIsMe = m.ballRetainer == hi;
        if (m.ballRetainer != -1 && !retainerIsMe) return -1;
        const lm::SinCosF bk = back(angle);
        Vec3 inMov = rotby(sp.movement, bk);
        int bestAnim = -1;
        Vec3 bestSmuggle2D;
        Vec3 desMov = desDir * desVel;
        float height = s.ctx.staticData->data[hi].height;
        const int ft = string_to_function_type(A(sorted[0]).animationType);
        float tmpRot = 0, predAngle = 0;
        Vec3 adOutMov;
        bool found = false;
        for (int entry = 0; entry < sorted.count && !found; entry++) {
            const int ai = sorted[entry];
            const Anim &a = A(ai);
            bool isBase = a.baseAnimation;
            physics_vector(ai, useDesMov, desMov, useDesBody, desBodyRel, posOut, tmpRot);
            predAngle = a.outgoingAngle.value() + tmpRot;
            predAngle = wrap_range(-kPi, kPi, predAngle);
            Vec3 outMov = rotby(outgoing_movement_of(posOut), bk);
            adOutMov = outMov;
            const int total = a.footballCount;
            if (total > 64) {
                s.fail(kStatusOverflow);
                return -1;
            }
            int touchIDs[64];
            int nt = 0;
            for (int tch = total / 2; tch > -1; tch--) touchIDs[nt++] = tch;
            for (int tch = total / 2 + 1; tch < total; tch++) touchIDs[nt++] = tch;
            int defTouch = D(ai).touchFrame;
            for (int tn = 0; tn < total && !found; tn++) {
                if (touchIDs[tn] >= total) {
                    s.fail(kStatusUnsupported);
                    return -1;
                }
                const FootballKey &fk = s.T().football[a.firstFootball + touchIDs[tn]];
                Vec3 animBall = fk.position;
                int atf = fk.frame;
                if (!retainerIsMe) {
                    Vec3 abs = ball_predict(m.ball, atf * 10);
                    if (fabsf(abs.c[0]) > kPitchHalfL + kLineHalfW + 0.11f ||
                        fabsf(abs.c[1]) > kPitchHalfW + kLineHalfW + 0.11f)
                        continue;
                }
                Vec3 touchMov = rotby(movement_at_frame(posOut.el, posOut.count, atf, 0), bk);
                Vec3 bpos = mental_ball_at(atf * 10);
                Vec3 bmov = (mental_ball_at(atf * 10 + 10) - mental_ball_at(atf * 10)) * 100.0f;
                bpos = rotby(bpos - sp.position, bk);
                bmov = rotby(bmov, bk);
                const Vec3 touchPos = rotby(posOut[atf], bk);
                Vec3 bodyPos = touchPos;
                bodyPos.c[2] = 0;
                Quat abr;
                Vec3 abp;
                float z;
                key_frame_z(s.T(), a, kBpPlayer, atf, abr, abp, z);
                float abh = animBall.c[2];
                animBall = (animBall - abp) + touchPos;
                animBall.c[2] = abh * (height / kPlayerHeight);
                {
                    Vec3 before = bpos - bmov * 0.006f;
                    Vec3 after = bpos + bmov * 0.003f;
                    float frac = clampf_(line_closest_to_point(before, after, animBall), 0.0f, 1.0f);
                    bpos = before + (after - before) * frac;
                }
                Vec3 sm3 = bpos - animBall;
                Vec3 sm2 = sm3.flat();
                float bdz = fabsf(sm3.c[2]);
                bdz *= 1.0f - clampf_((float)(((double)animBall.c[2] - 0.11) * (double)0.3f), 0.0f, 0.2f);
                bdz *= 1.0f - clampf_((float)(((double)bpos.c[2] - 0.11) * (double)0.4f), 0.0f, 0.3f);
                if (bpos.c[2] > 1.8f && bpos.c[2] > animBall.c[2] + 0.12f) bdz *= 2.0f;
                if (bpos.c[2] > 2.6f && bpos.c[2] > animBall.c[2] + 0.08f) bdz *= 20.0f;
                if (ft == kFtDeflect) bdz *= 0.8f;
                if (retainerIsMe) bdz = 0.0f;
                if (bpos.c[2] < 0.5f && isBase) bdz = std_max(bdz - 0.15f, 0.0f);
                if (bdz < 0.22f) {
                    int dtf = defTouch - atf;
                    float awk = nclamp((float)(dtf < 0 ? -dtf : dtf), 0.0f, 4.0f);
                    awk = awk * awk * 0.5f;
                    float tff = atf / 24.0f;
                    tff = lm::lm_powf(tff, 0.7f);
                    if (tff > 1.0f) tff = 1.0f + ((tff - 1.0f) * 0.5f);
                    float rco = 0.0f;
                    float rf = 0.3f * (1.0f - awk);
                    if (ft == kFtDeflect) { rf *= 1.8f; rco += 0.4f; }
                    if (ft == kFtSliding) { rf *= 0.2f; rco = 0.0f; }
                    if (ft == kFtInterfere) { rf *= 1.4f; rco += 0.2f; }
                    if (ft == kFtShortPass || ft == kFtLongPass || ft == kFtHighPass || ft == kFtShot) {
                        rf *= 1.3f;
                        rco += 0.15f;
                    }
                    if ((ft == kFtTrap || ft == kFtBallControl) && preferPassAndShot) rf *= 0.3f;
                    rco *= (1.0f - awk);
                    float tv = touchMov.length();
                    Vec3 foot = front_of_foot_offset(tv, z, bpos.c[2]);
                    if (vel_category(tv) != kVelIdle)
                        rot2d_inplace(foot, fix_angle(angle2d(touchMov.normalized(Vec3(0, -1, 0)))));
                    float ltb = curve(last_touch_bias_at(600, m.actualTime_ms + (uint64_t)(int64_t)(atf * 10)), 1.0f);
                    if (ltb > 0.0f) {
                        float f = 1.0f - ltb * 0.97f * (1.0f - stat(kStTechnicalBallControl) * 0.1f);
                        rf *= f;
                        rco *= f;
                    }
                    float trf = rf * tff;
                    float adv = body_ball_advantage(a, touchMov, inMov, adOutMov, predAngle, bodyPos, foot,
                                                    animBall.flat(), bpos.flat(), trf, rco);
                    if (adv >= 1.0f || retainerIsMe) {
                        found = true;
                        bestAnim = ai;
                        bestSmuggle2D = sm2;
                        touchFrameOut = atf;
                    }
                }
            }
        }
        if (found) {
            touchPosOut = mental_ball_at(touchFrameOut * 10);
            Vec3 full = rotby(bestSmuggle2D, turn(angle));
            smuggleOut = full;
            float sd = smuggleOut.length();
            float mul = 0.4f;
            if (ft != kFtBallControl) mul *= 0.8f;
            if (touchPosOut.c[2] > 0.5f) mul *= 0.7f;
            if (touchPosOut.c[2] > 1.0f) mul *= 0.7f;
            float bonus = 0.0f;
            if (ft == kFtInterfere) bonus += 0.1f;
            sd = clampf_(sd - (0.02f + bonus), 0.0f, (float)100.0);
            sd *= 1.0f - mul;
            sd = std_min(sd, smuggleOut.length() - 0.2f);
            if (retainerIsMe) sd = 0.0f;
            smuggleOut = smuggleOut.normalized(Vec3(0)) * sd;
            {
                float toStraight = angle + predAngle;
                rot2d_inplace(smuggleOut, -toStraight);
                float shorten = 0.02f;
                float allowFwd = 0.25f *
                                 (1.0f - lm::lm_powf(nclamp(adOutMov.length(), kIdleVel, kSprintVel - 2.0f), 0.6f)) *
                                 (touchFrameOut * 0.1f);
                if (ft != kFtBallControl && ft != kFtTrap) allowFwd += 0.1f;
                if (smuggleOut.c[1] < 0.0f) smuggleOut.c[1] = clampf_(smuggleOut.c[1] + shorten, -allowFwd, 0.0f);
                rot2d_inplace(smuggleOut, toStraight);
            }
            smuggleOut *= 0.7f + 0.3f * nclamp(closest_opponent_distance(s, hi), 0.6f, 1.2f);
        }
        rotSmuggleOut = tmpRot;
        return bestAnim;
    }

    // Common tail of both selections: make the chosen animation current.
    CB_HD void commit(int sel, const PlayerCommand &cmd, int interrupt, const PosList &pos, int touchFrame,
                      const Vec3 &touchPos, const Vec3 &smuggle, float rotSmuggle, float rotScale) {
        Humanoid &h = H();
        AnimationState &ca = h.anim;
        SpatialState &sp = SP();
        h.prevAnimFrameNumber = ca.frameNumber;
        h.prevAnimFunctionType = ca.functionType;
        const Anim &next = A(sel);
        ca.anim = sel;
        ca.id = sel;
        ca.functionType = cmd.desiredFunctionType;
        ca.frameNumber = 0;
        ca.touchFrame = touchFrame;
        ca.originatingInterrupt = interrupt;
        ca.touchPosition = touchPos;
        const float maxRot = 0.25f * kPi;
        set_radian(ca.rotationSmuggle.begin,
                   clampf_(wrap_range(-kPi, kPi, sp.relBodyAngleNonQuantized.value() - next.incomingBodyAngle.value()) * 1.0f,
                           -maxRot * rotScale, maxRot * rotScale));
        set_radian(ca.rotationSmuggle.end, rotSmuggle);
        set_radian(ca.rotationSmuggleOffset, 0);
        ca.actionSmuggle = smuggle;
        ca.actionSmuggleOffset = Vec3(0);
        ca.actionSmuggleSustain = Vec3(0);
        ca.actionSmuggleSustainOffset = Vec3(0);
        ca.movementSmuggle = Vec3(0);
        ca.movementSmuggleOffset = Vec3(0);
        ca.incomingMovement = sp.movement;
        ca.outgoingMovement = outgoing_movement_of(pos);
        ca.positions.count = pos.count;
        for (int i = 0; i < pos.count; i++) ca.positions[i] = pos[i];
        ca.positionOffset = Vec3(0);
        ca.originatingCommand = cmd;
    }

    CB_HD void pre_select_foot(int interrupt) {
        AnimationState &ca = H().anim;
        SpatialState &sp = SP();
        if (interrupt != kIntReQueue || ca.frameNumber > 12) {
            const Anim &cur = A(ca.anim);
            sp.foot = cur.outgoingFoot;
            if (cur.outgoingSpecialState != kSS_Empty) {
                sp.floatVelocity = 0;
                sp.velocityCategory = kVelIdle;
                sp.movement = Vec3(0);
            }
        }
    }

    CB_HDNI int base_select(const PlayerCommand &cmd, int interrupt);
    CB_HDNI int select(const PlayerCommand &cmd, int interrupt, bool preferPassAndShot);
};

// Officials and reset paths (GRF HumanoidBase::SelectAnimation).
CB_HDNI int Selector::base_select(const PlayerCommand &cmd, int interrupt) {
    Humanoid &h = H();
    AnimationState &ca = h.anim;
    SpatialState &sp = SP();
    const int ft = cmd.desiredFunctionType;
    pre_select_foot(interrupt);
    const Anim &cur = A(ca.anim);
    const float angle = sp.angle.value();
    CrudeQuery q;
    q.byFunctionType = true;
    q.functionType = ft;
    q.byIncomingVelocity = true;
    q.incomingVelocity = sp.velocityCategory;
    q.incomingVelocityStrict = true;
    q.byIncomingBodyDirection = true;
    q.incomingBodyDirectionStrict = true;
    q.incomingBodyDirection = sp.relBodyDirectionVector;
    q.incomingVelocityForceLinearity = true;
    q.incomingBodyDirectionForceLinearity = true;
    if (ft == kFtTrip) {
        q.byTripType = true;
        q.tripType = cmd.tripType;
    }
    q.incomingSpecialState = cur.outgoingSpecialState;
    if (s.w.m.ballRetainer == hi) q.incomingRetainState = D(ca.anim).outgoingRetainRawValue;
    if (cmd.useSpecialVar1) q.specialVar1 = (float)cmd.specialVar1;
    if (cmd.useSpecialVar2) q.specialVar2 = (float)cmd.specialVar2;
    if (cur.outgoingSpecialState != kSS_Empty) q.incomingVelocity = kVelIdle;
    AnimList l;
    crude_selection(s, q, l);
    if (l.count == 0) {
        if (ft == kFtMovement) l.push((int16_t)idle_movement_animation());
        else return kSelFalse;
    }
    float adDesVel = cmd.desiredVelocityFloat;
    if (cmd.useDesiredMovement) {
        Vec3 rel = rotby(cmd.desiredDirection, back(angle));
        set_movement_predicate(rel, vel_category(adDesVel));
        pr.lookAt = cmd.desiredLookAt;
        if (ft == kFtMovement) {
            keep_best_direction(l, cmd, true);
            if (cmd.useDesiredLookAt) keep_best_body_direction(l, cmd, true);
        } else {
            sort(l, [&](int i) { return movement_similarity_key(i); });
        }
    }
    pr.idle = 1;
    pr.desiredFoot = sp.foot;
    pr.relIncomingBodyDirection = sp.relBodyDirectionVector;
    pr.incomingVelocity = sp.velocityCategory;
    if (cmd.useDesiredTripDirection) pr.relDesiredTripDirection = rotby(cmd.desiredTripDirection, back(angle));
    int sel = -1;
    PosList tmpPos;
    float tmpRot = 0;
    if (l.count == 0) return kSelFalse;
    const bool byTrip = cmd.useDesiredTripDirection, byBase = ft != kFtMovement;
    const int qi = l.count > 1 ? incoming_body_query() : 0;
    const int firstAnim = first_of_chain(l, 4 + byTrip + byBase, [&](int i, double *k) {
        int n = 0;
        if (byBase) k[n++] = A(i).baseAnimation ? 0 : 1;
        if (byTrip) k[n++] = -D(i).bumpDirection.dot(pr.relDesiredTripDirection);
        k[n++] = key_incoming_velocity(A(i), pr);
        k[n++] = incoming_body_key(i, qi);
        k[n++] = key_foot(A(i), pr);
        k[n++] = key_idle(A(i), pr);
    });
    if (ft == kFtMovement || ft == kFtTrip || ft == kFtSpecial) {
        sel = firstAnim;
        const Anim &na = A(sel);
        Vec3 desMov = cmd.desiredDirection * cmd.desiredVelocityFloat;
        Vec3 desBodyRel = Vec3(0, -1, 0);
        if (cmd.useDesiredLookAt)
            desBodyRel = (rotby((cmd.desiredLookAt - sp.position).flat(), back(angle)) - na.translation)
                             .normalized(Vec3(0, -1, 0));
        physics_vector(sel, cmd.useDesiredMovement, desMov, cmd.useDesiredLookAt, desBodyRel, tmpPos, tmpRot);
    }
    if (interrupt == kIntReQueue && sel != -1 && ca.positions.count > 1 && tmpPos.count > 1) {
        const Anim &sa = A(sel);
        bool curIdle = vel_category(cur.outgoingVelocity) == kVelIdle;
        if (ca.functionType == ft &&
            ((!curIdle && cur.quadrantID == sa.quadrantID) ||
             (curIdle && fabsf(preferred_out_angle(ca.anim) - preferred_out_angle(sel)) < 0.20f * kPi)))
            sel = -1;
    }
    if (sel == -1) return kSelFalse;
    commit(sel, cmd, interrupt, tmpPos, -1, Vec3(), Vec3(), tmpRot, 1.0f);
    return kSelTrue;
}

CB_HDNI int Selector::select(const PlayerCommand &cmd, int interrupt, bool preferPassAndShot) {
    Player &pl = player();
    Humanoid &h = H();
    AnimationState &ca = h.anim;
    SpatialState &sp = SP();
    const MatchState &m = s.w.m;
    const int ft = cmd.desiredFunctionType;
    const bool retainerIsMe = m.ballRetainer == hi;
    if (ft != kFtMovement && ft != kFtTrip && ft != kFtSpecial && ft != kFtSliding) {
        if ((mental_ball_at(200).flat() - sp.position).length() > 10.0f) return kSelFalse;
        if ((mental_ball_at(kTouchOffset_ms).flat() - sp.position).length() > 2.0f &&
            (mental_ball_at(kTouchOffset_ms).flat() -
             (sp.position + sp.movement * (float)kTouchOffset_ms * (float)0.001))
                    .length() > (mental_ball_at(0).flat() - sp.position).length())
            return kSelFalse;
    }
    if (ft != kFtMovement && ft != kFtTrip && ft != kFtSpecial && ft != kFtSliding && ft != kFtDeflect &&
        !retainerIsMe) {
        if ((mental_ball_at(1000) - ball_predict(m.ball, 1000)).length() > 2.0f) return kSelFalse;
    }
    if (interrupt == kIntReQueue) {
        if (m.designatedPossessionPlayer < 0) return kSelUnsupported;
        float focusDist = (hum(s.w, m.designatedPossessionPlayer).spatial.position - sp.position).length();
        const int cft = ca.functionType;
        const int eff = A(ca.anim).frameCount - 1;
        if (cft != kFtMovement && ft == kFtMovement) return kSelFalse;
        if (cft == kFtMovement && ft == kFtMovement && (pl.hasPossession || focusDist > 12.0f)) return kSelFalse;
        if (cft == kFtMovement && ft == kFtMovement && ca.frameNumber + 6 > eff) return kSelFalse;
        if (cft == kFtMovement && ft == kFtMovement && h.requeueDelayFrames > 0) return kSelFalse;
        if (cft == kFtBallControl && ft == kFtBallControl && (ca.frameNumber > 8 || h.requeueDelayFrames > 0))
            return kSelFalse;
        if (cft == kFtBallControl && ft == kFtTrap) return kSelFalse;
        if (cft == kFtTrap && ft == kFtTrap && (ca.frameNumber + 6 > ca.touchFrame || h.requeueDelayFrames > 0))
            return kSelFalse;
        if (cft == kFtTrap && ft == kFtBallControl &&
            (ca.frameNumber + 6 > ca.touchFrame || h.requeueDelayFrames > 0))
            return kSelFalse;
        const PlayerCommand &oc = ca.originatingCommand;
        if (oc.desiredFunctionType == ft &&
            ((oc.desiredDirection * oc.desiredVelocityFloat) - (cmd.desiredDirection * cmd.desiredVelocityFloat)).length() <
                1.5f)
            return kSelFalse;
        if ((cft == kFtMovement && ft == kFtMovement) || (cft == kFtBallControl && ft == kFtBallControl) ||
            (cft == kFtTrap && ft == kFtBallControl) || (cft == kFtTrap && ft == kFtTrap)) {
            Vec3 planned = ca.outgoingMovement - ca.incomingMovement;
            Vec3 desired = (cmd.desiredDirection * cmd.desiredVelocityFloat) - sp.movement;
            if ((desired.dot(planned) > 0.0f && get_distance(desired, planned) < 4.0f) ||
                desired.dot(planned) > 0.8f || get_distance(desired, planned) < 2.0f)
                return kSelFalse;
        }
        if (cft == kFtMovement && ft == kFtBallControl &&
            (m.actualTime_ms - pl.base.lastTouchTime_ms < 600 && pl.base.lastTouchType == kTouchKicked) &&
            pl.hasPossession) {
            float dmc = (sp.movement - (cmd.desiredDirection * cmd.desiredVelocityFloat)).length();
            if (dmc < 1.0f) return kSelFalse;
        }
    }
    pre_select_foot(interrupt);
    const Anim &cur = A(ca.anim);
    const float angle = sp.angle.value();
    CrudeQuery q;
    q.byFunctionType = true;
    q.functionType = ft;
    if (q.functionType == kFtLongPass) q.functionType = kFtShortPass;
    if (cmd.touchInfo.desiredPower != 0.0f) {
        q.byOutgoingBallDirection = true;
        q.outgoingBallDirection = rotby(cmd.touchInfo.desiredDirection, back(angle));
    }
    q.byIncomingVelocity = true;
    q.incomingVelocity = sp.velocityCategory;
    if (q.functionType != kFtMovement && q.incomingVelocity == kVelDribble) q.incomingVelocity = kVelWalk;
    q.incomingVelocityStrict = false;
    if (q.functionType != kFtMovement && q.functionType != kFtBallControl) {
        q.incomingVelocityForceLinearity = false;
        if (q.functionType != kFtDeflect) {
            q.incomingVelocityNoDribbleToSprint = true;
            if (q.functionType != kFtShortPass && q.functionType != kFtLongPass &&
                q.functionType != kFtHighPass && q.functionType != kFtShot) {
                q.incomingVelocityForceLinearity = true;
                q.incomingVelocityNoDribbleToIdle = true;
            } else {
                q.incomingVelocityForceLinearity = false;
                q.incomingVelocityNoDribbleToIdle = false;
            }
        } else {
            q.incomingVelocityNoDribbleToSprint = false;
            q.incomingVelocityNoDribbleToIdle = false;
        }
    } else {
        q.incomingVelocityStrict = true;
    }
    q.byIncomingBodyDirection = true;
    q.incomingBodyDirection = sp.relBodyDirectionVector;
    if (q.functionType != kFtMovement) {
        q.incomingBodyDirectionStrict = false;
        if (q.functionType != kFtDeflect)
            q.incomingBodyDirectionForceLinearity = q.functionType != kFtBallControl;
        else
            q.incomingBodyDirectionForceLinearity = false;
    } else {
        q.incomingBodyDirectionStrict = true;
    }
    q.bySide = false;
    if (cmd.useDesiredLookAt && (cur.outgoingSpecialState == kSS_Empty) && !retainerIsMe) {
        Vec3 lav = (cmd.desiredLookAt - sp.position).normalized(sp.directionVector);
        q.lookAtVectorRelative = rotby(lav, back(angle));
        q.bySide = true;
    }
    if (cmd.onlyDeflectAnimationsThatPickupBall) {
        q.byPickupBall = true;
        q.pickupBall = true;
    }
    if (ft == kFtTrap || ft == kFtInterfere || ft == kFtDeflect) {
        q.byIncomingBallDirection = true;
        q.incomingBallDirection =
            rotby(mental_ball_at(180) - mental_ball_at(120), back(angle)).normalized(Vec3(0));
    }
    q.allowLastDitch = allow_last_ditch();
    if (ft == kFtTrip) {
        q.byTripType = true;
        q.tripType = cmd.tripType;
    }
    q.incomingSpecialState = cur.outgoingSpecialState;
    if (retainerIsMe) q.incomingRetainState = D(ca.anim).outgoingRetainRawValue;
    if (cmd.useSpecialVar1) q.specialVar1 = (float)cmd.specialVar1;
    if (cmd.useSpecialVar2) q.specialVar2 = (float)cmd.specialVar2;
    if (cur.outgoingSpecialState != kSS_Empty) q.incomingVelocity = kVelIdle;
    AnimList l;
    crude_selection(s, q, l);
    if (l.count == 0) {
        if (ft == kFtMovement) l.push((int16_t)idle_movement_animation());
        else return kSelFalse;
    }
    if (cmd.useDesiredMovement) {
        Vec3 rel = rotby(cmd.desiredDirection, back(angle));
        set_movement_predicate(rel, vel_category(cmd.desiredVelocityFloat));
        pr.lookAt = cmd.desiredLookAt;
        if (ft == kFtMovement) {
            keep_best_direction(l, cmd, true);
            if (cmd.useDesiredLookAt) keep_best_body_direction(l, cmd, true);
        } else if (ft == kFtBallControl) {
            bool strict = !allow_last_ditch();
            float allowed = 0.0f * kPi;
            if (cmd.useDesiredLookAt) keep_best_body_direction(l, cmd, strict, allowed);
            keep_best_direction(l, cmd, strict, allowed, 0);
        } else if (ft == kFtTrap) {
            bool hob = high_or_bouncy();
            bool strict = !(allow_last_ditch(false) || hob);
            float allowed = 0.3f * kPi;
            keep_best_direction(l, cmd, strict, allowed, 2, -1);
            if (cmd.useDesiredLookAt) keep_best_body_direction(l, cmd, strict, allowed);
            if (!high_or_bouncy() && q.allowLastDitch == false) {
                Vec3 desMov = cmd.desiredDirection * cmd.desiredVelocityFloat;
                const Anim &best = A(l[0]);
                Vec3 bestOut = rotby(best.outgoingMovement, turn(angle));
                float cdd = cmd.desiredDirection.dot(sp.directionVector);
                bool allow = true;
                float ad = fabsf(angle2d_to(rotby(best.outgoingDirection, turn(angle)), cmd.desiredDirection));
                if (ad > 0.375f * kPi) allow = false;
                Vec3 dbd = bestOut - desMov;
                if ((dbd.length() > kWalkVel + 0.5f && cdd > 0.0f) || (dbd.length() > kSprintVel + 0.5f && cdd <= 0.0f))
                    allow = false;
                if (!allow) return kSelFalse;
            }
        } else if (ft == kFtInterfere) {
            bool strict = cmd.strictMovement == kStrictTrue;
            float allowed = 0.3f * kPi;
            keep_best_direction(l, cmd, strict, allowed, 1);
            if (cmd.useDesiredLookAt) keep_best_body_direction(l, cmd, strict, allowed);
        }
    }
    const bool firstOnly = ft == kFtMovement || ft == kFtTrip || ft == kFtSpecial;
    if (!firstOnly) sort(l, [&](int i) { return D(i).priorityAbsolute; });
    int desiredIdle = 0;
    if (!m.inPlay) desiredIdle = 2;
    if (m.inSetPiece) desiredIdle = 1;
    else if ((ball_predict(m.ball, 200) - sp.position).length() > 16.0f) desiredIdle = 1;
    pr.idle = (float)desiredIdle;
    if (!firstOnly) sort(l, [&](int i) { return key_idle(A(i), pr); });
    pr.desiredFoot = sp.foot;
    if (!firstOnly) sort(l, [&](int i) { return key_foot(A(i), pr); });
    if (ft != kFtBallControl) {
        pr.relIncomingBodyDirection = sp.relBodyDirectionVector;
        if (!firstOnly) sort_incoming_body(l);
    }
    pr.incomingVelocity = sp.velocityCategory;
    if (!firstOnly) sort(l, [&](int i) { return key_incoming_velocity(A(i), pr); });
    if (cmd.useDesiredTripDirection) {
        pr.relDesiredTripDirection = rotby(cmd.desiredTripDirection, back(angle));
        if (!firstOnly) sort(l, [&](int i) { return -D(i).bumpDirection.dot(pr.relDesiredTripDirection); });
    }
    if (ft != kFtMovement && !firstOnly) sort_base(l);
    if (ft == kFtDeflect) sort(l, [&](int i) { return D(i).outgoingRetainRaw ? 0 : 1; });
    int sel = -1;
    PosList tmpPos;
    int tmpTouch = -1;
    Vec3 tmpTouchPos, tmpSmuggle;
    float tmpRot = 0;
    if (l.count == 0 && ft == kFtMovement) l.push((int16_t)idle_movement_animation());
    Vec3 desBodyRel = Vec3(0, -1, 0);
    if (cmd.useDesiredLookAt)
        desBodyRel = rotby((cmd.desiredLookAt - (sp.position + sp.movement * 0.1f)).normalized(Vec3(0, -1, 0)),
                           back(angle));
    if (firstOnly) {
        const bool byTrip = cmd.useDesiredTripDirection, byBase = ft != kFtMovement;
        const int qi = l.count > 1 ? incoming_body_query() : 0;
        sel = first_of_chain(l, 5 + byTrip + byBase, [&](int i, double *k) {
            int n = 0;
            if (byBase) k[n++] = A(i).baseAnimation ? 0 : 1;
            if (byTrip) k[n++] = -D(i).bumpDirection.dot(pr.relDesiredTripDirection);
            k[n++] = key_incoming_velocity(A(i), pr);
            k[n++] = incoming_body_key(i, qi);
            k[n++] = key_foot(A(i), pr);
            k[n++] = key_idle(A(i), pr);
            k[n++] = D(i).priorityAbsolute;
        });
        Vec3 desMov = cmd.desiredDirection * cmd.desiredVelocityFloat;
        physics_vector(sel, cmd.useDesiredMovement, desMov, cmd.useDesiredLookAt, desBodyRel, tmpPos, tmpRot);
    } else if (ft == kFtBallControl) {
        if (need_touch(l[0], cmd))
            sel = best_cheatable(l, cmd.useDesiredMovement, cmd.desiredDirection, cmd.desiredVelocityFloat,
                                 cmd.useDesiredLookAt, desBodyRel, tmpPos, tmpTouch, tmpTouchPos, tmpSmuggle, tmpRot,
                                 preferPassAndShot);
    } else if (ft == kFtTrap || ft == kFtInterfere || ft == kFtDeflect) {
        sel = best_cheatable(l, cmd.useDesiredMovement, cmd.desiredDirection, cmd.desiredVelocityFloat,
                             cmd.useDesiredLookAt, desBodyRel, tmpPos, tmpTouch, tmpTouchPos, tmpSmuggle, tmpRot,
                             preferPassAndShot);
    } else if (ft == kFtShortPass || ft == kFtLongPass || ft == kFtHighPass || ft == kFtShot) {
        sel = best_cheatable(l, cmd.useDesiredMovement, cmd.desiredDirection, cmd.desiredVelocityFloat,
                             cmd.useDesiredLookAt, desBodyRel, tmpPos, tmpTouch, tmpTouchPos, tmpSmuggle, tmpRot);
    } else if (ft == kFtSliding) {
        sel = best_cheatable(l, cmd.useDesiredMovement, cmd.desiredDirection, cmd.desiredVelocityFloat,
                             cmd.useDesiredLookAt, desBodyRel, tmpPos, tmpTouch, tmpTouchPos, tmpSmuggle, tmpRot);
        if (sel == -1 && l.count > 0) {
            sel = l[0];
            Vec3 desMov = cmd.desiredDirection * cmd.desiredVelocityFloat;
            physics_vector(sel, cmd.useDesiredMovement, desMov, cmd.useDesiredLookAt, desBodyRel, tmpPos, tmpRot);
        }
    }
    if (interrupt == kIntReQueue && sel != -1 && ca.positions.count > 1 && tmpPos.count > 1) {
        const Anim &sa = A(sel);
        bool curIdle = vel_category(cur.outgoingVelocity) == kVelIdle;
        bool selIdle = vel_category(sa.outgoingVelocity) == kVelIdle;
        if (ca.functionType == ft &&
            ((!curIdle && cur.quadrantID == sa.quadrantID) ||
             ((curIdle && selIdle) && fabsf(preferred_out_angle(ca.anim) - preferred_out_angle(sel)) < 0.06f * kPi)))
            sel = -1;
    }
    if (sel == -1) return kSelFalse;
    const float rotScale = ft == kFtMovement ? 1.0f : 0.5f;
    commit(sel, cmd, interrupt, tmpPos, tmpTouch, tmpTouchPos, tmpSmuggle, tmpRot, rotScale);
    ca.movementSmuggle = movement_smuggle();
    ca.movementSmuggleOffset = Vec3(0);
    return kSelTrue;
}

}  // namespace cb
