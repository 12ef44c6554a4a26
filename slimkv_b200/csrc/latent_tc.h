// Launch interface of the tcgen05 latent-branch attention (latent_tc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace slimkv {

struct TcJob {
    int rank_k, rank_v, kchunks, vchunks;
    const int32_t* seqlens;   // latents per sequence
    const int32_t* qlens;     // queries per sequence (1 or 2), nullable
    int length;
    float scale_log2;
    int splits, tiles_per_split;
    int rows_alloc, out_width;
    float* part_o;            // [B][splits][rows_alloc][out_width]
    float* part_lse;          // [B][splits][rows_alloc]
    unsigned int* status;
};

struct TcLaunch {
    int batch, length, rank_k, rank_v, width, lat_capacity;
    const void* lat_k;
    const void* lat_v;
    int64_t lat_stride_batch, lat_stride_row;   // elements
    const void* q_hilo;                          // [B][128][width] bf16: row hl*32*nq + l*32 + head, hl 0 = hi, 1 = lo
    const int32_t* latent_len;
    const int32_t* query_len;
    float scale;
    int splits, tiles_per_split, rows_alloc;
    float* part_o;
    float* part_lse;
    unsigned int* status;
};

constexpr int kTcTileKeys = 128;

int launch_latent_tc(const TcLaunch& launch, cudaStream_t stream);

}  // namespace slimkv
