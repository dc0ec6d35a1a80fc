/*
 * mlvc_oracle — CPU restatement of the reference's per-operator arithmetic
 * for the FP16 convolution stack.  TEST INFRASTRUCTURE ONLY: tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg use it as the
 * checker; the product never links, loads or calls it.
 *
 * All tensors are NCHW, FP16 stored as raw uint16 bits, math in FP32 with one
 * FP16 rounding per graph operator, exactly where the reference rounds:
 *   conv      backends/cpu/src/kernels_scalar.cpp:112-196 (accumulator starts
 *             at the bias, FP32 multiply-add over (ky, kx, ic), one rounding)
 *             and backends/driver_cubin/kernels/generic_conv.cu:1-82 (groups)
 *   unary     backends/driver_cubin/kernels/elementwise.cu:59-79
 *   binary    backends/driver_cubin/kernels/elementwise.cu:23-45 (4-D
 *             broadcast by size-1 dimensions)
 * FP16 conversion is IEEE-754 binary16 with round-to-nearest-even, restated
 * from the standard (the reference's core/include/mlvc/core/half.hpp does the
 * same in software).
 */
#ifndef MLVC_ORACLE_H
#define MLVC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float oracle_half_to_float(uint16_t h);
uint16_t oracle_float_to_half(float f);
void oracle_halves_to_floats(const uint16_t* src, float* dst, size_t n);
void oracle_floats_to_halves(const float* src, uint16_t* dst, size_t n);

/* Grouped 2-D convolution with symmetric padding; bias may be NULL.
 * epilogue: 0 none, 1 LeakyReLU(alpha), 2 residual add (residual NCHW, same
 * shape as the output).  The epilogue runs on the already-rounded conv value
 * and rounds again (kernels_scalar.cpp:180-192). */
void oracle_conv2d(const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                   uint16_t* y, int n, int ic, int ih, int iw, int oc, int oh,
                   int ow, int kh, int kw, int sh, int sw, int ph, int pw,
                   int groups, int epilogue, float alpha,
                   const uint16_t* residual);

/* op: 0 LeakyReLU, 1 Clip, 2 Sigmoid, 3 Reciprocal, 4 Round. */
void oracle_unary(const uint16_t* x, uint16_t* y, size_t count, int op,
                  float alpha, float lo, float hi);

/* op: 0 Add, 1 Mul, 2 Sub.  od/ad/bd are 4-D shapes (rank-padded with 1s). */
void oracle_binary(const uint16_t* a, const uint16_t* b, uint16_t* y,
                   const int64_t* od, const int64_t* ad, const int64_t* bd,
                   int op);

#ifdef __cplusplus
}
#endif
#endif
