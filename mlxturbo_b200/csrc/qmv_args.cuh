// qmv_args.cuh -- argument block of the decode/gather kernel (qmv.cu).
#pragma once

#include <stdint.h>

namespace qmm {

// Gather description: rows sorted by expert, 16-row items.
struct Segments {
    const int32_t* row_start;    // [E+1]
    const int32_t* tile_prefix;  // [E+1], items of up to 16 rows per expert
    const uint32_t* row_src;     // x row of sorted row s, or null (s)
    const uint32_t* row_dst;     // output row of sorted row s, or null (s)
    const float* row_scale;      // output scale of sorted row s, or null
    int E;
    int x_rows;                  // rows of x: a gathered row outside [0, x_rows) reads zeros
    int y_rows;                  // rows of y: a scattered row outside [0, y_rows) is not stored
    long long w_stride;          // words per expert
    long long s_stride;          // scales per expert
};

struct QmvArgs {
    const uint16_t* x;
    const uint32_t* w;
    const uint16_t* sc;
    const uint16_t* bi;
    uint16_t* y;
    int M, N, K;
    Segments seg;
};

}  // namespace qmm
