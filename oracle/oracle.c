/*
 * oracle.c -- CPU restatement of the three recurrent operators of
 * XMetAI-Lab/xmetai-onnx-plugins. TEST INFRASTRUCTURE: only the tests,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs load
 * this library, and only as a checker or a timed CPU baseline. The product
 * (libxm_ops.so) never links or calls it.
 *
 *   oracle_*_f64: golden restatement, FP64 state and accumulation, libm
 *                 exp/log1p/tanh/sin/cos. Used as the parity reference.
 *   oracle_*_f32: the same token-sequential recurrence in FP32 (the
 *                 "sequential C++ CPU recurrence" baseline), OpenMP-parallel over
 *                 independent (batch, channel) / (batch, head) units.
 *
 * Parity of this restatement is pinned against the reference kernels
 * themselves: oracle/ref_driver.cu runs the reference CUDA sources rebuilt for
 * sm_100a and tests/golden/make_golden.py stores their outputs as fixtures.
 */
#include <math.h>
#include <stddef.h>
#include <stdlib.h>

#define REAL double
#define OUT_T double
#define FN(name) name##_f64
#define EXP exp
#define LOG1P log1p
#define SQRT sqrt
#define TANH tanh
#define SIN sin
#define COS cos
#define FLOOR floor
#include "oracle_impl.h"
#undef REAL
#undef OUT_T
#undef FN
#undef EXP
#undef LOG1P
#undef SQRT
#undef TANH
#undef SIN
#undef COS
#undef FLOOR

#define REAL float
#define OUT_T float
#define FN(name) name##_f32
#define EXP expf
#define LOG1P log1pf
#define SQRT sqrtf
#define TANH tanhf
#define SIN sinf
#define COS cosf
#define FLOOR floorf
#include "oracle_impl.h"

int oracle_version(void) { return 1; }
