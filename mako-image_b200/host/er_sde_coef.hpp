// The scalar part of one ER-SDE step (ErSde::step, src/image/er_sde.cpp:27-74), shared by the host step and the
// device step so both use the same double-precision coefficients.
#pragma once

#include "mkb_image.h"

namespace mkb {

struct ErSdeCoef {
    int stage = 1;      // 1..3: how many previous image estimates enter the update
    bool last = false;  // sigma_{i+1} == 0: the step lands on the image estimate
    double c1 = 0, c2 = 0, c3 = 0, c4 = 0, d_den = 1, u_den = 1, cn = 0;
};

// Coefficients of step i with noise scale s_noise; false if i is out of range.
bool er_sde_coef(const mkb_er_sde* e, int i, float s_noise, ErSdeCoef* c);
// The level sigma_i of step i in double precision (after the flow model's first-level substitution).
double er_sde_sigma_d(const mkb_er_sde* e, int i);
// Device-step bookkeeping: true if step i may run now (i == 0 starts a run; otherwise it must follow i - 1).
bool er_sde_dev_order(mkb_er_sde* e, int i);

}  // namespace mkb
