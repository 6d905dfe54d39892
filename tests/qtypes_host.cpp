// Host build of tier_b200/csrc/tk_qtypes.h -- the same element decode the
// dequant and GEMV kernels run -- so tests/test_qtypes_host.py can hold it
// against the golden vectors and the reference's q_val on the CPU.
#include <stddef.h>
#include "tk_qtypes.h"

extern "C" int tkq_host_geom(int t, int* elems, int* bytes) {
    *elems = tkq::elems(t);
    *bytes = tkq::bytes(t);
    return *elems > 0;
}

extern "C" void tkq_host_dequant(const uint8_t* W, size_t row_bytes, int t, int rows, int cols, float* out) {
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) out[(size_t)r * cols + c] = tkq::value(W + (size_t)r * row_bytes, t, c);
}

extern "C" float tkq_host_half(unsigned h) { return tkq::half_to_f32(h); }
