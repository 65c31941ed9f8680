// tcgen05 GEMM interface (see gemm.cu).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace rf {

enum GemmEpilogue : int { kEpiStore = 0, kEpiSwiGLU = 1, kEpiF32 = 2, kEpiF64Acc = 3, kEpiPeer = 4, kEpiNvlsAR = 5, kEpiNvlsAG = 6 };

constexpr int kMaxPeers = 8;

// Peer-store epilogue (kEpiPeer): bf16 tiles written straight into other GPUs' buffers (CUDA IPC mappings).
//  mode 0 (scatter to row owner): rows are split in n_peers chunks of row_chunk; the tile of row r goes to
//          peer[r / row_chunk] + slot * slot_stride + (r % row_chunk) * ld + col
//  mode 1 (broadcast): every peer gets the tile at peer[q] + r * ld + col_off + col
struct PeerArgs {
  void* peer[kMaxPeers];
  int n_peers;
  int mode;
  int slot;
  int row_chunk;
  long slot_stride;
  long ld;
  long col_off;
};

// Fused all-reduce through NVSwitch multicast (kEpiNvlsAR): the epilogue stores this rank's partial tile into its
// symmetric partial buffer (args.out, residual added when given) and counts finished tiles per 128-row block; the
// last tile of a block announces it to every rank. Two extra warps per CTA (the comm warps) take the row blocks
// this rank owns (mb % world == rank) as soon as every rank has announced them, reduce them in the switch
// (multimem.ld_reduce) and multicast the sums (multimem.st) into every rank's output buffer; a final barrier
// makes the whole result visible on every rank before the kernel ends.
// Fused all-gather through NVSwitch multicast (kEpiNvlsAG, the column-sharded map fill): args.out is the
// multicast address of the full [M][ldo] buffer already offset to this rank's first column; every 16-byte store
// of the epilogue (bias added) lands in every rank's copy; a final barrier (done flags at index
// max_mb * kMaxPeers + rank) makes the gathered tensor complete on every rank before the kernel ends.
struct NvlsGemmArgs {
  const void* mc_part;      // multicast address of the partial buffer (bf16 [M][ldo])
  void* mc_out;             // multicast address of the output buffer
  int* flags;               // this rank's flag words: [row block][rank] epochs, then done[rank]
  int* peer_flags[kMaxPeers];
  int world, rank, epoch;
  int* rb_count;            // local per-row-block tile counters (zero between launches)
  int* done_count;          // local CTA counter (zero between launches)
  int max_mb;               // row blocks the flag array holds
  int comm_off;             // diagnostics: announce and barrier but move no data (times the GEMM part alone)
  int comm_ctas;            // > 0: that many trailing CTAs only reduce (the others only compute tiles)
};

struct GemmOperands {
  const void* A;   // bf16; [M, K] (K-major) or [K, M] (MN-major), row pitch lda elements
  long lda;
  bool a_mn;
  const void* B;   // bf16; [N, K] (K-major) or [K, N] (MN-major), row pitch ldb elements
  long ldb;
  bool b_mn;
};

struct GemmArgs {
  int M, N, K;
  int k_splits;                     // split-K chunks (fp64 epilogue only); 1 otherwise
  int k_chunk;                      // K elements per chunk (multiple of 64)
  void* out;                        // bf16 / fp32 / fp64 by epilogue
  long ldo;                         // output row pitch in elements
  const __nv_bfloat16* bias;        // [N] or nullptr (kEpiStore)
  const __nv_bfloat16* residual;    // [M, N] or nullptr (kEpiStore); may alias out
  long ldr;
  int vec_ok;                       // out/residual pitches and bases allow 16-byte vector access
  int* err;                         // device error word (bounded waits), may be nullptr
  PeerArgs peer;                    // kEpiPeer only
  NvlsGemmArgs nvls;                // kEpiNvlsAR only
};

void gemm_bf16(const GemmOperands& op, GemmArgs args, int epi, int bn, int max_ctas, cudaStream_t stream);
// gemm2sm.cu: the two-SM (cta_group::2, 256 x 256 tile) kernel for K-major store / SwiGLU products with M >= 256;
// returns false (nothing launched) for any other call. gemm_bf16 tries it first for 256-column tiles.
// max_ctas >= 2: at most max_ctas / 2 clusters (the rest of the SMs stay free for a kernel on another stream)
bool gemm_bf16_2sm(const GemmOperands& op, const GemmArgs& args, int epi, int max_ctas, cudaStream_t stream);
extern bool gemm_2sm_enabled;
// gemv.cu: products of 1-16 rows (K-major operands, store / SwiGLU / fp32 epilogues) as bandwidth-bound GEMVs;
// false (nothing launched) for any other call. gemm_bf16 tries it first.
bool gemm_bf16_gemv(const GemmOperands& op, const GemmArgs& args, int epi, int bn, cudaStream_t stream);
extern bool gemv_enabled;
extern bool gemv_mma;       // true: the tensor-core kernel (1-16 rows); false: the CUDA-core kernel (1-8 rows)
extern int gemv_max_rows;   // products of up to this many rows take the GEMV
CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t pitch_elems,
                              uint32_t box_inner, uint32_t box_outer);
int num_sms(int device);

}  // namespace rf
