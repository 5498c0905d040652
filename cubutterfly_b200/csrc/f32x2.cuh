// f32x2.cuh -- packed fp32 pairs on Blackwell's f32x2 pipe.
//
// Two fp32 lanes live in one 64-bit register pair; add/sub/mul/fma.rn.f32x2
// operate on both lanes with one instruction (same IEEE rounding per lane as
// the scalar forms).
#pragma once

#include "common.cuh"

namespace cubf::f32x2 {

using P = unsigned long long;  // two fp32 lanes

CUBF_DEV P pk(float lo, float hi) {
    P r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
CUBF_DEV void up(P p, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(p)); }
CUBF_DEV P add2(P a, P b) {
    P r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
CUBF_DEV P sub2(P a, P b) {
    P r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
CUBF_DEV P mul2(P a, P b) {
    P r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
CUBF_DEV P fma2(P a, P b, P c) {
    P r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

}  // namespace cubf::f32x2
