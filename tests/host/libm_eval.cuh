// Test infrastructure: one evaluation of the library's restatement of a glibc math function
// (cuju_b200/csrc/libm.cuh), widened to double, numbered as oracle/units.cpp's oracle_libm numbers
// the reference's: 0 sinf, 1 cosf, 2 powf, 3 acosf, 4 asinf, 5 atanf, 6 atan2f (y, x), 7 sin, 8 cos,
// 9 acos, 10 pow, 11 the sine of sincosf, 12 its cosine, 13 the positive-base powf.
#pragma once

#include "libm.cuh"

CB_HD double libm_eval(int which, double x, double y) {
    const float xf = (float)x, yf = (float)y;
    switch (which) {
        case 0: return cb::lm::lm_sinf(xf);
        case 1: return cb::lm::lm_cosf(xf);
        case 2: return cb::lm::lm_powf(xf, yf);
        case 3: return cb::lm::lm_acosf(xf);
        case 4: return cb::lm::lm_asinf(xf);
        case 5: return cb::lm::lm_atanf(xf);
        case 6: return cb::lm::lm_atan2f(yf, xf);
        case 7: return cb::lm::lm_sin(x);
        case 8: return cb::lm::lm_cos(x);
        case 9: return cb::lm::lm_acos(x);
        case 10: return cb::lm::lm_pow(x, y);
        case 11: return cb::lm::lm_sincosf(xf).s;
        case 12: return cb::lm::lm_sincosf(xf).c;
        case 13: return cb::lm::lm_powf_pos(xf, yf);
    }
    return 0.0;
}
