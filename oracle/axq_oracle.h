/*
 * CPU oracle for the block-quantized matmul path — TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference's CPU algorithms for
 * quantize / dequantize / quantized matmul (ruwwww/Axon,
 * src/backend/cpu_backend.cpp).  It exists to check the CUDA product
 * path; nothing in the product links, loads or calls it.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may use it.
 *
 * Parity pinning: the restatement is checked byte-for-byte against the
 * reference compiled from its own sources (oracle/Makefile -> oracle/_ref)
 * and against the golden fixtures under tests/golden/ generated from that
 * build (tests/golden/make_golden.py).
 *
 * Format ids are the reference's QuantFormat ordinals
 * (include/axon/core/types.h:36-45).
 */
#ifndef AXQ_ORACLE_H
#define AXQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ORC_NONE = 0, ORC_Q8_0 = 1, ORC_Q6_K = 2, ORC_Q5_K = 3,
    ORC_Q4_0 = 4, ORC_Q4_K = 5, ORC_Q3_K = 6, ORC_Q2_K = 7
};

uint16_t orc_float_to_half(float f);
float orc_half_to_float(uint16_t h);

/* Bytes of one block and elements per block; 0 for an unknown format. */
size_t orc_block_bytes(int fmt);
int orc_block_elems(int fmt);
/* quantized_size (cpu_backend.cpp:693) and quantized_size_2d (:713). */
size_t orc_quantized_size(size_t numel, int fmt);
size_t orc_quantized_size_2d(int64_t rows, int64_t cols, int fmt);

/* Row-wise pack of src[rows x cols] (cpu_backend.cpp:1171-1257).  A 1-D
 * tensor of n elements is rows=1, cols=n (:1259-1329).  Returns 0 on
 * success, -1 for an unknown format. */
int orc_quantize(int fmt, const float* src, int64_t rows, int64_t cols, void* dst);
/* Row-wise decode (cpu_backend.cpp:1334-1670). */
int orc_dequantize(int fmt, const void* src, int64_t rows, int64_t cols, float* dst);
/* out[M x N] = A_q[M x K] . B[K x N], the scalar loops of
 * cpu_backend.cpp:1674-2066 (fp32 sequential accumulation).  Q8_0 has no
 * reference kernel: it follows matmul_q4's loop with the Q8_0 decode. */
int orc_matmul(int fmt, const void* a_q, const float* b, float* out,
               int64_t M, int64_t K, int64_t N);
/* Same product, computed from the dequantized weights in double precision
 * (a tighter yardstick for kernels that reorder the fp32 sum). */
int orc_matmul_f64(int fmt, const void* a_q, const float* b, double* out,
                   int64_t M, int64_t K, int64_t N);
/* As orc_matmul over rows [row0, row1) of A_q only (for threaded timing). */
int orc_matmul_rows(int fmt, const void* a_q, const float* b, float* out,
                    int64_t M, int64_t K, int64_t N, int64_t row0, int64_t row1);

#ifdef __cplusplus
}
#endif
#endif
