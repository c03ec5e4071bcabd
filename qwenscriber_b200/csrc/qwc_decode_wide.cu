// qwc_decode_wide.cu -- the persistent decode kernel of qwc_decode.cu with a
// weight ring of three 57 KB slots instead of five of 34 KB.
//
// With K = 6144 (the 1.7B decoder's down projection) a CTA's 14 rows of down
// weights are 45.7 KB: two narrow tiles, one wide tile; gate and up take two
// wide tiles instead of three narrow ones. Models whose stages already fit
// narrow slots keep the deeper five-slot prefetch (qwc_api.cpp chooses). The
// slot layout is a compile-time constant in both copies: a run-time slot count
// measured slower in every configuration.

#define QWC_DECODE_WIDE_SLOTS 1
#include "qwc_decode.cu"
