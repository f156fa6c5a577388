// ref_shim_tables.cpp -- exposes the reference's full iq2_xxs tables.
// TEST INFRASTRUCTURE ONLY (oracle/_ref).  The upstream RVV kernel's
// tables.h:8-108 holds the 256-entry lattice and the 128x8 even-sign table;
// they pin the grid encoding used by the oracle and the kernels.
#include <cstdint>

#include "tables.h"

extern "C" {
uint64_t ref_iq2xxs_grid_upstream(unsigned index) { return iq2xxs_grid[index & 255u]; }
int ref_keven_signs_q2xs(unsigned index) { return keven_signs_q2xs[index & 1023u]; }
}
