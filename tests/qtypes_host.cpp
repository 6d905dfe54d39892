// Host build of tier_b200/csrc/tk_qtypes.h -- the same element decode the
// dequant and GEMV kernels run -- so tests/test_qtypes_host.py can hold it
// against the golden vectors and the reference's q_val on the CPU.
#include <stddef.h>
#include "tk_qgrid.h"
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

// Lattice types: `tab` is a tkq::GRID_BYTES buffer with the grids at their
// offsets; tkq_host_fill_signs writes the sign table the library builds.
extern "C" int tkq_host_grid_bytes(int t) { return tkq::grid_bytes(t); }
extern "C" int tkq_host_grid_offset(int which) {
    const int off[7] = {tkq::GRID_IQ2XXS, tkq::GRID_IQ2XS, tkq::GRID_IQ2S, tkq::GRID_IQ3XXS,
                        tkq::GRID_IQ3S,   tkq::GRID_IQ1S,  tkq::GRID_SIGNS};
    return which >= 0 && which < 7 ? off[which] : tkq::GRID_BYTES;
}
extern "C" void tkq_host_fill_signs(int8_t* tab) {
    for (int i = 0; i < 128; ++i) tab[tkq::GRID_SIGNS + i] = (int8_t)tkq::sign_byte(i);
}
extern "C" void tkq_host_dequant_grid(const uint8_t* W, size_t row_bytes, int t, int rows, int cols,
                                      const int8_t* tab, float* out) {
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c)
            out[(size_t)r * cols + c] = tkq::grid_value(W + (size_t)r * row_bytes, t, c, tab);
}
