// Launchers of the non-GEMM sm_100a kernels. Raw pointers + a stream; no torch types.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include <atomic>
#include <mutex>
#include <string>
#include <utility>

namespace rf {

// Runs a set-up step once per CUDA device (the current one) for one call site, safely from several host threads.
// Function attributes such as the dynamic shared-memory limit belong to a device, so every device a process
// launches on needs its own cudaFuncSetAttribute.
struct PerDeviceOnce {
  static constexpr int kMaxDevices = 64;
  std::once_flag flag[kMaxDevices];
  template <class F>
  void operator()(F&& f) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
      f();
      return;
    }
    std::call_once(flag[dev], std::forward<F>(f));
  }
};

// Writes `code` into a device error word the way the kernels do (first error wins), in the stream's order.
void record_error_async(int* err, int code, cudaStream_t stream);

// Host-side count of kernel launches issued by this library (bench.py reports it per timed region).
inline std::atomic<long>& launch_counter() {
  static std::atomic<long> c{0};
  return c;
}
inline void count_launch(long n = 1) { launch_counter().fetch_add(n, std::memory_order_relaxed); }

// ---- norm.cu
void rmsnorm(const __nv_bfloat16* x, long ldx, const __nv_bfloat16* w, __nv_bfloat16* y, long ldy, int rows, int d,
             float eps, int zero_centred, cudaStream_t stream);

struct HeadNormRopeArgs {
  const __nv_bfloat16* src;   // head h of row t at src + t * src_row_stride + h * src_head_stride
  long src_row_stride;
  long src_head_stride;
  int n_heads, head_dim, n_rows;
  const __nv_bfloat16* norm_w;  // [head_dim] or nullptr
  int norm_mode;                // -1 none, 0 plain RMSNorm, 1 zero-centred
  float eps;
  const __nv_bfloat16* cos;     // [max_pos, rot / 2] bf16 tables
  const __nv_bfloat16* sin;
  int rot;                      // rotated dims (0: no RoPE)
  const int* pos;               // [n_rows] positions, or nullptr: row + pos_offset
  int pos_offset;
  __nv_bfloat16* dst;           // head h of row t at dst + h * dst_head_stride + t * dst_row_stride
  long dst_head_stride;
  long dst_row_stride;
  // paged destination (dst_pages != nullptr): row t goes to cache row r = dst_row0 + t, stored in page
  // dst_pages[r / page_size] at dst + page * dst_page_stride + h * dst_head_stride + (r % page_size) * dst_row_stride
  const int* dst_pages = nullptr;
  int page_size = 0;
  long dst_page_stride = 0;
  int dst_row0 = 0;
  // dst_row_from_pos: source row t goes to cache row pos[t] (positions read on the device: a decode step captured in
  // a CUDA graph writes at the position held in device memory); rows >= dst_rows (the capacity) are not written
  int dst_row_from_pos = 0;
  int dst_rows = 0;
};
void head_norm_rope(const HeadNormRopeArgs& a, cudaStream_t stream);

void gated_rmsnorm(const __nv_bfloat16* o, long ldo, const __nv_bfloat16* z, long ldz, const __nv_bfloat16* w,
                   __nv_bfloat16* y, long ldy, int rows, int heads, int dv, float eps, cudaStream_t stream);

void embed_gather(const __nv_bfloat16* table, const int64_t* ids, __nv_bfloat16* out, int rows, int d, long vocab,
                  cudaStream_t stream,
                  int* err = nullptr);

// ---- attention.cu
struct AttnArgs {
  const __nv_bfloat16* q;   // [hq, nq, hd] (head-major; row pitch hd, head pitch q_head_stride)
  long q_head_stride;
  const __nv_bfloat16* k;   // [hkv, *, hd] cache (head pitch kv_head_stride, row pitch hd)
  const __nv_bfloat16* v;
  long kv_head_stride;
  int hq, hkv, hd, nq, nk;
  const int* qpos;          // [nq] sorted query positions, or nullptr: q_start + row
  int q_start;
  float scale;
  const __nv_bfloat16* gate;   // optional output gate: gate of (row t, head h) at gate + t * gate_row + h * gate_head
  long gate_row, gate_head;
  __nv_bfloat16* out;          // [nq, hq * hd] (row pitch out_row)
  long out_row;
  int* err;                    // bounded-wait error word (tcgen05 path)
  int impl;                    // 0 auto (tcgen05 when possible), 1 mma.sync kernel, 2 tcgen05 only
  // paged K/V (kv_pages != nullptr, tcgen05 path only): k / v point at pools [num_pages][hkv][page_size][hd]; key row
  // j lives in page kv_pages[j / page_size] at row j % page_size; page_size a multiple of the key tile (128)
  const int* kv_pages = nullptr;
  int page_size = 0;
  int num_pages = 0;
};
void flash_attention(const AttnArgs& a, cudaStream_t stream);
bool flash_attention_tc(const AttnArgs& a, cudaStream_t stream);
extern int attn_p_buffers;   // 1 or 2 shared-memory P buffers in the tcgen05 attention (2 by default)
extern int attn_poly;         // 0, 2 or 4 of every 8 softmax exponentials on the FMA pipe (exp2_fma)
extern int attn_softmax_groups;   // softmax warpgroups of the tcgen05 attention (1 or 2; 1 by default)
extern int attn_s_buffers;        // TMEM S buffers of the tcgen05 attention (2 or 3; 0: per head dim)
extern int attn_q_tmem;           // 1: the tcgen05 attention's S product reads Q from TMEM (A operand)
extern int attn_rotate;           // 1: every CTA of the tcgen05 attention walks the key tiles from its own start

// ---- gdn.cu
struct GdnPrepArgs {
  const __nv_bfloat16* proj;   // [n, *] in-projection rows: [q | k | v] conv channels at col 0, b at b_off, a at a_off
  long proj_row;
  int b_off, a_off;
  const __nv_bfloat16* conv_w;  // [C, K]
  const __nv_bfloat16* conv_state;  // [K-1, C] previous pre-conv rows (zeros at the start)
  const float* A_log;           // [nv]
  const float* dt_bias;         // [nv]
  int n, nk, nv, dk, dv, K;
  __nv_bfloat16* q;             // [nk, n, dk] l2-normed, scaled by dk^-0.5 (nullptr: fill mode, q heads skipped)
  __nv_bfloat16* k;             // [nk, n, dk] l2-normed
  __nv_bfloat16* v;             // [nv, n, dv]
  float* beta;                  // [nv, n]
  float* g;                     // [nv, n]
};
void gdn_prep(const GdnPrepArgs& a, cudaStream_t stream);
// gdn_decode.cu: one decode row of a GDN layer for up to kDecodeSeqs sequences (conv, gates, recurrent delta-rule
// step, conv-state shift); sequence s of the launch reads in-projection row r0 + s and writes output row r0 + s.
constexpr int kDecodeSeqs = 16;
struct GdnDecodeArgs {
  const __nv_bfloat16* proj;     // [R, *] in-projection rows: [q | k | v] conv channels at col 0, b at b_off, a at a_off
  long proj_row;
  int b_off, a_off;
  const __nv_bfloat16* conv_w;   // [C, K]
  const float* A_log;            // [nv]
  const float* dt_bias;          // [nv]
  int nk, nv, dk, dv, K;
  __nv_bfloat16* out;            // [R, nv * dv]
  long out_row;
  const __nv_bfloat16* conv_src[kDecodeSeqs];   // [K-1, C] per sequence
  __nv_bfloat16* conv_dst[kDecodeSeqs];
  const float* rec_src[kDecodeSeqs];            // [nv, dk, dv] fp32 per sequence
  float* rec_dst[kDecodeSeqs];
};
bool gdn_decode_supported(int dk, int dv, int K);
constexpr int kDecSplits = 64;   // key splits per (sequence, KV head) of the decode attention, at most
// attention_decode.cu: one decode row of an attention layer for up to kDecodeSeqs sequences (K/V append at the
// row of each sequence's device position, q / k head norm + RoPE, split-key attention, combine); sequence s of the
// launch reads projected row r0 + s, position pos[r0 + s], and writes output row r0 + s.
struct DecodeAttnArgs {
  const __nv_bfloat16* qkv;      // [R, *]: q heads (each [q | gate] when gated) | k heads | v heads
  long qkv_row;
  int hq, hkv, hd, gated;
  const __nv_bfloat16* q_norm;   // [hd] or nullptr
  const __nv_bfloat16* k_norm;
  int norm_mode;                 // -1 none, 0 plain RMSNorm, 1 zero-centred
  float eps;
  const __nv_bfloat16* cos;      // [max_pos, rot / 2] bf16 tables
  const __nv_bfloat16* sin;
  int rot;
  const int* pos;                // [R] positions; the new K/V row of a sequence is cache row pos
  float scale_log2;              // softmax scale times log2(e)
  __nv_bfloat16* out;            // [R, hq * hd]
  long out_row;
  float* part_o;                 // [R, hkv, kDecSplits, G, hd] fp32 split partials
  float* part_ml;                // [R, hkv, kDecSplits, G, 2] (max, sum)
  int* err;
  __nv_bfloat16* k[kDecodeSeqs];          // contiguous: [hkv, rows, hd] buffers; paged: the pool's K / V
  __nv_bfloat16* v[kDecodeSeqs];
  const int* pages[kDecodeSeqs];          // page table of the sequence, or nullptr (contiguous)
  int rows[kDecodeSeqs];                  // rows the sequence's cache can hold
  long head_stride[kDecodeSeqs];          // elements between KV heads (contiguous: rows * hd; paged: page_size * hd)
  int page_size;
  long page_stride;
};
bool decode_attention_supported(int hd, int hq, int hkv, int rot);
void decode_attention(const DecodeAttnArgs& a, int r0, int rows, cudaStream_t stream);
void gdn_decode_step(const GdnDecodeArgs& a, int r0, int rows, cudaStream_t stream);
void gdn_conv_state_update(const __nv_bfloat16* proj, long proj_row, __nv_bfloat16* state, int n, int C, int K,
                           cudaStream_t stream);

struct GdnScanArgs {
  const __nv_bfloat16* q;   // [nk, n, dk] (nullptr: fill mode, no output)
  const __nv_bfloat16* k;   // [nk, n, dk]
  const __nv_bfloat16* v;   // [nv, n, dv]
  const float* beta;        // [nv, n]
  const float* g;           // [nv, n]
  float* state;             // [nv, dk, dv] fp32, read and updated in place
  __nv_bfloat16* out;       // [n, nv, dv] (row pitch out_row) or nullptr
  long out_row;
  __nv_bfloat16* w_buf;     // scratch [nv, n_pad, dk]
  __nv_bfloat16* u_buf;     // scratch [nv, n_chunks, dv, 64]: U^T per chunk
  __nv_bfloat16* s_buf;     // scratch [nv, n_chunks, dv, dk]: chunk-start S^T (output mode)
  __nv_bfloat16* vt_buf;    // scratch [nv, n_chunks, dv, 64]: V'^T per chunk (output mode)
  int n, nk, nv, dk, dv;
  int* err;
  int groups;               // > 1: two-level scan over this many chunk groups (dk == dv); else sequential
  float* grp_buf;           // scratch [2][nv][groups][dv][dk]: per group the end state from zero (R) and the
                            // transfer matrix (P), both in the transposed-state layout
  float* start_buf;         // scratch [nv][groups][dv][dk]: group-start S^T (output mode)
};
void gdn_chunk_scan(const GdnScanArgs& a, cudaStream_t stream);
extern int gdn_fused_output;   // 1 (default): output mode in the state pass; 0: state pass + separate output pass
// gdn_tc.cu: the output-mode state pass (sequential, mode 0, or the two-level scan's pass 3, mode 2) on tcgen05 with
// the state in TMEM; false when the shapes do not fit it (dk = dv = 128) or it is switched off (gdn_state_tc = 0,
// the default: measured slower than the mma.sync pass)
bool gdn_state_out_tc(const GdnScanArgs& a, int n_pad, int mode, cudaStream_t stream);
extern int gdn_state_tc;
extern unsigned long long* gdn_tc_trace;   // [chunks][16] ns phase stamps of the first CTA, or nullptr

// ---- moe.cu
void router_topk(const float* logits, long ld, int n, int E, int k, int* idx, float* wts, int norm,
                 cudaStream_t stream);
void moe_align(const int* idx, int n, int k, int e0, int E, int* counts, int* rank, int* seg_start, int* tile_start,
               int* pos, const __nv_bfloat16* x, long ldx, __nv_bfloat16* xp, int d, cudaStream_t stream);
void grouped_gemm(const __nv_bfloat16* xp, long rows_cap, const __nv_bfloat16* w, int E, int N, int K,
                  const int* seg_start, const int* tile_start, __nv_bfloat16* out, long ldo, int swiglu, int* err,
                  cudaStream_t stream);
void moe_combine(const __nv_bfloat16* h, long ldh, const __nv_bfloat16* y, const int* pos, const float* w, int n,
                 int k, const __nv_bfloat16* ys, const float* gate_logit, long ldg, __nv_bfloat16* out, int d,
                 cudaStream_t stream);

// ---- linalg.cu
void cholesky_solve(double* a, int n, long lda, double shift, double* b, long ldb, int R, int* err, cudaStream_t s);

// vocabulary reductions of fp32 logits rows: lse (fp64), argmax, target log-prob, KL(ref || logits)
struct ScoreArgs {
  const float* logits;
  long ld;
  int rows, V;
  const float* ref;       // optional reference rows (KL, reference argmax)
  long ld_ref;
  const long* targets;    // optional [rows]
  double* logprob;        // [rows] (with targets)
  double* lse;            // optional [rows]
  int* argmax;            // optional [rows]
  int* ref_argmax;        // optional [rows]
  double* kl;             // optional [rows] (with ref)
};
void score_rows(const ScoreArgs& a, cudaStream_t stream);

// reduce.cu: read cosine of the lambda selection, window attention mass of the selectors
void row_cosine(const __nv_bfloat16* a, long lda, const __nv_bfloat16* b, long ldb, long rows, int d, float eps,
                float* out, cudaStream_t stream);
struct WindowMassArgs {
  const __nv_bfloat16* q;     // window queries [hq][w][hd] (post-RoPE)
  long q_head_stride, q_row_stride;
  const __nv_bfloat16* k;     // keys [hkv][n][hd] (post-RoPE, as cached)
  long k_head_stride, k_row_stride;
  const int* qpos;            // [w] positions of the window rows
  int hq, hkv, w, n, hd;
  float scale;
  float* part_m;              // scratch [hq * w][key blocks]
  float* part_l;
  float* qm;                  // scratch [hq * w]
  float* ql;
  double* mass;               // [n], accumulated
};
void window_mass(const WindowMassArgs& a, cudaStream_t stream);

// NVSwitch multicast collectives (nvls.cu). Flag words: slot * kMaxRanks + source rank, epoch-stamped.
constexpr int kMaxRanksNvls = 8;
struct NvlsFlags {
  int* local;                 // this rank's flag array
  int* peer[kMaxRanksNvls];   // every rank's flag array (unicast mappings, this rank's own included)
  int world, rank;
};
struct NvlsAllReduceArgs {
  const void* mc_in;                // multicast address of the partial rows (bf16 [rows][d])
  void* mc_out;                     // multicast address of the output rows
  const __nv_bfloat16* out_local;   // this rank's output buffer (unicast)
  __nv_bfloat16* dst;               // fresh [rows][d] result (nullptr: leave it in the output buffer)
  int rows, d, row0, row1;
  NvlsFlags f;
  int slot_in, slot_out, epoch;
  int* counter;                     // local grid counter (zero between launches)
  int* err;
  int max_ctas;                     // 0: one CTA per SM
  int acc32;                        // accumulate in fp32 in the switch (else bf16)
};
struct NvlsAllGatherArgs {
  const __nv_bfloat16* src;         // this rank's column slice [rows][cols], row pitch ld_src
  long ld_src;
  void* mc_out;                     // multicast address of the full [rows][d] buffer
  int rows, cols, d, col_off;
  NvlsFlags f;
  int slot, epoch;
  int* counter;
  int* err;
};
struct NvlsAllReduceF64Args {
  const void* mc_in;                // multicast address of every rank's fp64 vector [n]
  void* mc_out;                     // multicast address of the output vectors
  long n;
  NvlsFlags f;
  int slot_in, slot_out, epoch;
  int* counter;
  int* err;
};
void nvls_allreduce(const NvlsAllReduceArgs& a, cudaStream_t stream);
void nvls_allreduce_f64(const NvlsAllReduceF64Args& a, cudaStream_t stream);
void nvls_allgather(const NvlsAllGatherArgs& a, cudaStream_t stream);
void nvls_barrier(const NvlsFlags& f, int slot, int epoch, int* err, cudaStream_t stream);

// ---- comm.cu (peer-memory collectives; pointers are CUDA IPC mappings of the peers' buffers)
constexpr int kMaxRanks = 8;

struct PeerFlags {
  int* ptr[kMaxRanks];   // every rank's flag array (this rank's own included)
  int n;
};

struct ReduceRowsArgs {
  const __nv_bfloat16* recv;       // [n_peers slots][rows][d] partials of this rank's row block
  long slot_stride;                // elements between slots
  const __nv_bfloat16* residual;   // [rows][d] (row pitch ld_res) or nullptr
  long ld_res;
  __nv_bfloat16* red;              // [rows][d] reduced rows (this rank's IPC buffer)
  int rows, d, n_peers, my_rank;
  const int* flags;                // this rank's flag array
  int arrive_slot;                 // flags[arrive_slot + s]: rank s's partials have arrived
  int reduced_slot;                // flags[reduced_slot + q]: owner q's rows are reduced (set on every rank)
  int value;                       // the epoch of this call
  int* counter;                    // zero-initialised completion counter (this rank)
  PeerFlags peer_flags;
  int* err;
};

struct GatherRowsArgs {
  const __nv_bfloat16* peer_red[kMaxRanks];   // every owner's reduced rows
  int n_peers, row_chunk, total_rows, d;
  __nv_bfloat16* out;              // [total_rows][d] (row pitch ld_out)
  long ld_out;
  const int* flags;
  int reduced_slot;
  int value;
  int* err;
};

void comm_signal(const PeerFlags& f, int slot, int value, cudaStream_t stream);
// limit_ns: the wait's wall-time limit (0: the default, 10 s); on expiry kErrTimeoutPeer is recorded in err.
void comm_wait(const int* flags, int first, int n, int value, int* err, cudaStream_t stream, uint64_t limit_ns = 0);
void comm_reduce_rows(const ReduceRowsArgs& a, cudaStream_t stream);
void comm_gather_rows(const GatherRowsArgs& a, cudaStream_t stream);
void* ipc_malloc(size_t bytes);
void ipc_free(void* p);
std::string ipc_handle(void* p);
void* ipc_open(const std::string& handle);
void ipc_close(void* p);

}  // namespace rf
