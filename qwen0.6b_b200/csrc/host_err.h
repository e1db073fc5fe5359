// Internal host helpers shared by the translation units of libqwen_b200.so.
#pragma once
#include <cuda.h>

extern "C" {
// The thread-local error slot behind qwen_b200_last_error() (decode.cu).
void qb200_clear_error(void);
int qb200_set_error(int code, const char *msg);
}

// Tensor map of a 2-D fp16 row-major tensor [outer, inner] (row pitch in
// elements), box {box_inner, box_outer}; 128-byte swizzle when swizzle128.
// Returns 0 or an error code with the message recorded (ops.cu).
int qb200_encode_f16_2d(CUtensorMap *m, const void *ptr, long long inner, long long outer,
                        long long pitch, int box_inner, int box_outer, int swizzle128);
