// Launchers of the Q8_0 kernels (quantise, dequantise, split-KV decode).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gtb {

struct DecodeArgs {
    const void* q;
    int q_dtype;
    const void* k;
    const void* v;
    const int32_t* lens;
    int64_t B, H, Hkv, Smax, D;
    float scale;  // resolved (> 0)
    void* out;
    int* status;  // device status word for bounded waits
};

int launch_q8_0_quantize(const void* x, int x_dtype, int64_t nblocks, void* out, cudaStream_t st);
int launch_q8_0_dequantize(const void* blocks, int64_t nblocks, void* out, int out_dtype, cudaStream_t st);
// KV-cache append (x (B, Hkv, n_new, D) into cache rows pos[b] .. pos[b] + n_new - 1), then pos += n_new
// when `advance` (a second kernel, so every row's destination is read before it changes)
// (rope: rotate each new row for its cache position first; nullptr for none)
struct RopeArgs;
int launch_q8_0_append(const void* x, int x_dtype, int64_t B, int64_t Hkv, int64_t n_new, int64_t D, void* cache,
                       int64_t Smax, int32_t* pos, bool advance, const RopeArgs* rope, cudaStream_t st);
// RoPE of rows (rows = B*H*S of D values, position pos[row % S]) into out (rope.cu)
int launch_rope(const void* x, int dtype, int64_t rows, int64_t S, int64_t D, const int32_t* pos, const RopeArgs& r,
                void* out, cudaStream_t st);
// (cos, sin) table of n positions (rope.cu): tab[2 (s n_dims/2 + i)] = cos, sin of pair i at pos[s],
// as the rope kernels form the angles (the table of the tcgen05 forward's in-kernel rotation of q)
int launch_rope_table(const int32_t* pos, int64_t n, const RopeArgs& r, float* tab, cudaStream_t st);
int64_t decode_num_chunks(int64_t Smax);
// Scratch of one decode call: a work area of decode_work_bytes() for the persistent kernels (item
// counter, per-sequence item prefix [B + 1], per-sequence prefix of full-chunk items [B + 1], and at
// int offset decode_list_offset(B) the item list (full chunks first, then last partial chunks by
// decreasing size):
// one int2 (b, hk << 16 | chunk) per item), then the split-KV partials [B][Hkv][nchunks][G][D + 2] f32.
int64_t decode_list_offset(int64_t B);
size_t decode_work_bytes(int64_t B, int64_t Hkv, int64_t Smax);
size_t decode_scratch_bytes(int64_t B, int64_t H, int64_t Hkv, int64_t Smax, int64_t D);
int launch_decode_q8_0(const DecodeArgs& a, void* scratch, cudaStream_t st);

// tcgen05 decode (decode_sm100.cu): D = 128, f16 q, H/Hkv in {1, 2, 4, 8}, even Smax, 16-byte
// aligned q/k/v. Launches the plan kernel and the persistent kernel; partials as above.
bool decode_sm100_supported(const DecodeArgs& a);
int launch_decode_sm100(const DecodeArgs& a, int* work, float* part, int64_t nchunks, cudaStream_t st);
// Plan kernel of both persistent decode kernels: per-sequence item prefix, item list, zeroed counter.
int launch_decode_plan(const DecodeArgs& a, int* work, cudaStream_t st);

// Warp-MMA decode (decode_mma.cu): D = 128, f16 q, H/Hkv in {1, 2, 4}, even Smax, 16-byte aligned
// q/k/v. Same work area and partials as the tcgen05 kernel.
bool decode_mma_supported(const DecodeArgs& a);
int launch_decode_mma(const DecodeArgs& a, int* work, float* part, int64_t nchunks, cudaStream_t st);

}  // namespace gtb
