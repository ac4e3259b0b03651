// cuju-b200: GRF's quaternion and the angle helpers of its 3-vector, which call the glibc-exact
// transcendental functions of libm.cuh (cuju include/cuju/quaternion.h, vector3.h:185-231).
#pragma once

#include "libm.cuh"

namespace cb {

// 2-D rotation of a vector by an angle's cosine and sine (GRF Vector3::GetRotated2D).
CB_HD Vec3 rot2d_cs(const Vec3 &v, float cs, float sn) {
    Vec3 r;
    r.c[0] = (v.c[0] * cs) - (v.c[1] * sn);
    r.c[1] = (v.c[1] * cs) + (v.c[0] * sn);
    r.c[2] = v.c[2];
    return r;
}
CB_HD Vec3 rot2d(const Vec3 &v, float angle) {
    lm::SinCosF t = lm::lm_sincosf(angle);
    return rot2d_cs(v, t.c, t.s);
}
CB_HD void rot2d_inplace(Vec3 &v, float angle) {
    Vec3 r = rot2d(v, angle);
    v.c[0] = r.c[0];
    v.c[1] = r.c[1];
}
// GRF Vector3::GetAngle2D(): in [0, 2pi).
CB_HD float angle2d(const Vec3 &v) {
    float a = lm::lm_atan2f(v.c[1], v.c[0]);
    if (a < 0) a += 2 * kPi;
    return a;
}
// GRF Vector3::GetAngle2D(test): signed angle from v to test in [-pi, pi].
CB_HD float angle2d_to(const Vec3 &v, const Vec3 &t) {
    float a = -lm::lm_atan2f(v.c[0] * t.c[1] - v.c[1] * t.c[0], v.c[0] * t.c[0] + v.c[1] * t.c[1]);
    return wrap_range(-kPi, kPi, a);
}
CB_HD float distance(const Vec3 &a, const Vec3 &b) { return (a - b).length(); }

// GRF's quaternion: x, y, z then w.
struct Quat {
    float e[4];
    CB_HD Quat() : e{0, 0, 0, 1} {}
    CB_HD Quat(float x, float y, float z, float w) : e{x, y, z, w} {}
    CB_HD static Quat identity() { return Quat(0, 0, 0, 1); }
    CB_HD bool operator==(const Quat &o) const {
        return e[0] == o.e[0] && e[1] == o.e[1] && e[2] == o.e[2] && e[3] == o.e[3];
    }
    CB_HD bool operator!=(const Quat &o) const { return !(*this == o); }
    CB_HD void set(float x, float y, float z, float w) { e[0] = x; e[1] = y; e[2] = z; e[3] = w; }
    CB_HD Quat operator*(float s) const { return Quat(e[0] * s, e[1] * s, e[2] * s, e[3] * s); }
    CB_HD Quat operator*(const Quat &o) const {
        Quat p;
        p.e[0] = e[3] * o.e[0] + e[0] * o.e[3] + e[1] * o.e[2] - e[2] * o.e[1];
        p.e[1] = e[3] * o.e[1] + e[1] * o.e[3] + e[2] * o.e[0] - e[0] * o.e[2];
        p.e[2] = e[3] * o.e[2] + e[2] * o.e[3] + e[0] * o.e[1] - e[1] * o.e[0];
        p.e[3] = e[3] * o.e[3] - e[0] * o.e[0] - e[1] * o.e[1] - e[2] * o.e[2];
        return p;
    }
    // Rotates a vector with two cross products (GRF's form, exact only at unit length).
    CB_HD Vec3 operator*(const Vec3 &v) const {
        Vec3 q(e[0], e[1], e[2]);
        Vec3 c1 = q.cross(v);
        Vec3 c2 = q.cross(c1);
        c1 *= (2.0f * e[3]);
        c2 *= 2.0f;
        return v + c1 + c2;
    }
    CB_HD Quat operator+(const Quat &o) const {
        return Quat(e[0] + o.e[0], e[1] + o.e[1], e[2] + o.e[2], e[3] + o.e[3]);
    }
    CB_HD Quat operator-() const { return Quat(-e[0], -e[1], -e[2], -e[3]); }
    CB_HD void scale(float s) { for (int i = 0; i < 4; i++) e[i] *= s; }
    CB_HD float magnitude() const {
        if (e[0] == 0.0f && e[1] == 0.0f && e[2] == 0.0f && e[3] == 0.0f) return 0.0f;
        float m = sqrtf(e[0] * e[0] + e[1] * e[1] + e[2] * e[2] + e[3] * e[3]);
        if (m < kAboveMicro) return 0.0f;
        return m;
    }
    CB_HD Quat inverse() const {
        float m = magnitude();
        if (m < 0.000001f) return identity();
        float im = 1.0f / m;
        return Quat(-e[0] * im, -e[1] * im, -e[2] * im, e[3] * im);
    }
    // GRF's fast normalization: 2/(1+s) near unit length, 1/sqrt(s) otherwise; s summed in float,
    // the factor computed in double.
    CB_HD void normalize() {
        const float s = e[0] * e[0] + e[1] * e[1] + e[2] * e[2] + e[3] * e[3];
        if (s < 0.000001f)
            set(0, 0, 0, 1);
        else if (s < 2.0f || !(s <= 0x1p31f))
            scale((float)(2.0 / (1.0 + (double)s)));
        else
            scale((float)(1.0 / sqrt((double)s)));
    }
    CB_HD Quat normalized() const { Quat t(*this); t.normalize(); return t; }
    CB_HD float sq_magnitude() const { return e[0] * e[0] + e[1] * e[1] + e[2] * e[2] + e[3] * e[3]; }
    CB_HD float dot(const Quat &o) const {
        return e[0] * o.e[0] + e[1] * o.e[1] + e[2] * o.e[2] + e[3] * o.e[3];
    }
    CB_HD Quat rotation_to(const Quat &to) const { return to * inverse(); }
    CB_HD float rotation_angle(const Quat &to) const {
        return 2.0f * lm::lm_acosf(clampf_(dot(to), -1.0f, 1.0f));
    }
    CB_HD void set_angle_axis(float angle, const Vec3 &axis) {
        float half = 0.5f * angle;
        lm::SinCosF t = lm::lm_sincosf(half);
        e[0] = t.s * axis.c[0];
        e[1] = t.s * axis.c[1];
        e[2] = t.s * axis.c[2];
        e[3] = t.c;
    }
    CB_HD Quat lerp(float bias, const Quat &to) const {
        return (*this * (1 - bias) + to * bias).normalized();
    }
    CB_HD float same_neighborhood(const Quat &o) {
        float d = dot(o);
        if (d < 0) {
            d = -d;
            *this = -*this;
        }
        return d;
    }
    // Spherical interpolation: the dot sums in float (w, x, y, z), the rest in double.
    CB_HDNI Quat slerp(float bias, const Quat &to) const {
        Quat r;
        Quat t = to;
        double ch = e[3] * t.e[3] + e[0] * t.e[0] + e[1] * t.e[1] + e[2] * t.e[2];
        if (ch < 0) {
            t = -t;
            ch = -ch;
        }
        if (fabs(ch) >= 1.0) return *this;
        double sh = sqrt(1.0 - ch * ch);
        if (fabs(sh) < 0.000001f) {
            r.e[3] = (float)(e[3] * 0.5 + t.e[3] * 0.5);
            r.e[0] = (float)(e[0] * 0.5 + t.e[0] * 0.5);
            r.e[1] = (float)(e[1] * 0.5 + t.e[1] * 0.5);
            r.e[2] = (float)(e[2] * 0.5 + t.e[2] * 0.5);
            return r;
        }
        double half = lm::lm_acos(ch);
        const double af = (1 - bias) * half, at = bias * half;
        // sin(+-0) is that zero; skipping the call keeps the sign.
        double rf = (af == 0.0 ? af : lm::lm_sin(af)) / sh;
        double rt = (at == 0.0 ? at : lm::lm_sin(at)) / sh;
        r.e[3] = (float)(e[3] * rf + t.e[3] * rt);
        r.e[0] = (float)(e[0] * rf + t.e[0] * rt);
        r.e[1] = (float)(e[1] * rf + t.e[1] * rt);
        r.e[2] = (float)(e[2] * rf + t.e[2] * rt);
        return r;
    }
    CB_HDNI void angle_axis(float &angle, Vec3 &axis) const {
        angle = 2.0f * lm::lm_acosf(e[3]);
        float hs = sqrtf(1.0f - e[3] * e[3]);
        if (hs < 0.000001f) {
            axis.c[0] = e[0]; axis.c[1] = e[1]; axis.c[2] = e[2];
        } else {
            axis.c[0] = e[0] / hs; axis.c[1] = e[1] / hs; axis.c[2] = e[2] / hs;
        }
    }
    CB_HD Quat rotation_scaled(float factor) const {
        Quat r;
        Vec3 axis;
        float angle;
        angle_axis(angle, axis);
        if (angle > kPi) angle -= 2.0f * kPi;
        angle = fmodf(angle * factor, 2.0f * kPi);
        r.set_angle_axis(angle, axis);
        return r.normalized();
    }
    // GRF's Euler angles, with the y and z roles swapped; the singularity test in double.
    CB_HDNI void angles(float &ax, float &ay, float &az) const {
        const int X = 0, Y = 2, Z = 1;
        float test = e[X] * e[Y] + e[Z] * e[3];
        if ((double)test > 0.49999 || (double)test < -0.49999) {
            if (test > 0) {
                az = 2 * lm::lm_atan2f(e[X], e[Z]);
                ay = (float)((double)kPi * 0.5);
            }
            if (test < 0) {
                az = -2 * lm::lm_atan2f(e[X], e[Z]);
                ay = (float)((double)-kPi * 0.5);
            }
            ax = 0;
            return;
        }
        float sx = e[X] * e[X], sy = e[Y] * e[Y], sz = e[Z] * e[Z];
        az = lm::lm_atan2f(2 * e[Y] * e[3] - 2 * e[X] * e[Z], 1 - 2 * sy - 2 * sz);
        ay = lm::lm_asinf(2 * e[X] * e[Y] + 2 * e[Z] * e[3]);
        ax = lm::lm_atan2f(2 * e[X] * e[3] - 2 * e[Y] * e[Z], 1 - 2 * sx - 2 * sz);
    }
    CB_HDNI void set_angles(float ax, float ay, float az) {
        double s, c;
        s = lm::lm_sin((double)ay / 2.0); c = lm::lm_cos((double)ay / 2.0);
        float cy = (float)c, sy = (float)s;
        s = lm::lm_sin((double)az / 2.0); c = lm::lm_cos((double)az / 2.0);
        float cz = (float)c, sz = (float)s;
        s = lm::lm_sin((double)ax / 2.0); c = lm::lm_cos((double)ax / 2.0);
        float cx = (float)c, sx = (float)s;
        float cyz = cy * cz, syz = sy * sz;
        e[3] = cyz * cx - syz * sx;
        e[0] = cyz * sx + syz * cx;
        e[1] = sy * cz * cx + cy * sz * sx;
        e[2] = cy * sz * cx - sy * cz * sx;
    }
};

CB_HD Quat angle_axis_quat(float angle, const Vec3 &axis) {
    Quat q;
    q.set_angle_axis(angle, axis);
    return q;
}

}  // namespace cb
