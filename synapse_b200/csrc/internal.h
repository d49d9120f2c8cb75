// Entry points shared inside the library (not part of the public C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

// GGUF blocks of `rows` rows (device) -> rows [row0, row0 + rows) of a planar
// matrix of `total_rows` rows at dst.
int syn_repack_rows(int type, const void* src, int rows, int cols, void* dst, int total_rows, int row0,
                    cudaStream_t s);

// Random N(0, sigma) values, seeded by (seed, tensor, element), quantized with
// ggml's reference quantizer (Q4_0 / Q8_0) into rows [row0, row0 + rows) of a
// planar matrix of total_rows, or written as F32 / F16 (row0 must be 0).
int syn_fill_random(int type, int rows, int cols, void* dst, int total_rows, int row0, uint64_t seed,
                    uint64_t tensor, float sigma, cudaStream_t s);
// dst[i] = v for n floats.
int syn_fill_f32(float* dst, size_t n, float v, cudaStream_t s);

// Device-side greedy step bookkeeping (io layout in session.cpp): records the
// argmax, advances the position and picks the next input token.
int syn_advance(int32_t* io, const int32_t* forced, int32_t* history, cudaStream_t s);

// Programmatic dependent launch for this thread's launches.
void syn_set_pdl(int on);

// Sets the thread's last error message.
void syn_set_error(const char* msg);
