// Weight-streaming GEMV/GEMM-by-rows for the [out, in] weight layout, with fused prologue and
// epilogues. Host-side launch helpers are declared here and used by ops.cu and model.cu.
#pragma once

#include "runtime.h"

namespace l0b {

enum GemvEpi : int {
    EPI_STORE = 0,   // out[m, n - seg_begin] = y (+ bias)
    EPI_ACCUM = 1,   // out[m, n] += y               (residual add, f32 out)
    EPI_SWIGLU = 2,  // W = [gate; up] stacked: out[m, i] = silu(y[i]) * y[i + N/2]
    EPI_ARGMAX = 3,  // store logits (optional) and fold argmax into a 64-bit key per row
    EPI_PEER_SUM = 4  // out[m, n] += sum over the TP ranks, in rank order, of their y[m, n] (PeerSum below)
};

// All-reduce epilogue of a row-split projection under tensor parallelism (EPI_PEER_SUM, the tensor-core
// GEMV only). Each rank owns a peer-sum mailbox in its HBM, mapped into every rank by CUDA IPC:
//   data [2 parities][kMaxPeerRanks][kPeerSumSlotElems]  the ranks' partial outputs, [m][n], each one
//                                                        64-bit word (epoch << 32 | f32 bits)
// followed in the own mailbox by two counters: the epoch (fused calls completed) and the CTAs done in
// the current call. All ranks launch the same grid, so CTA c handles the same tiles everywhere: it
// stores its tiles' partials, tagged with the call's epoch, into its rank's slot of every mailbox (one
// 64-bit store per value: value and tag arrive together, so no fence and no separate flag), then reads
// the same elements of every rank's slot in its own mailbox -- waiting (bounded) until each carries
// the epoch -- and adds them to `out` in rank order: identical bits on every rank. The parity is the
// call's epoch & 1 (one epoch per call for every CTA: the last CTA to finish advances it), so a rank
// one call ahead writes the other half while a peer still reads this one; two calls ahead is
// impossible because finishing a call needs every rank's values of it, which each rank writes only
// after its previous call has completed (stream order).
constexpr int kMaxPeerRanks = 8;
constexpr int kPeerSumCtas = 1024;                   // CTAs of one fused launch at most
constexpr long long kPeerSumSlotElems = 1LL << 17;  // 8 rows of 16384
constexpr size_t kPeerSumDataBytes = 2ull * kMaxPeerRanks * kPeerSumSlotElems * sizeof(unsigned long long);
constexpr size_t kPeerSumBytes = kPeerSumDataBytes + 256;  // + epoch, done

struct PeerSum {
    char* mbox[kMaxPeerRanks];  // every rank's peer-sum mailbox in this process's address space
    int nranks, rank;
    int* error;  // device error flag, set when a wait gives up
};

struct GemvSeg {
    void* out;          // output base
    const float* bias;  // f32 [segment width] or null
    int row_end;        // exclusive end of this segment in W's rows (SWIGLU: in output columns)
    int ld;             // output row stride in elements
};

// Blocked int8 weight layout (kb > 0): [N / 16][K / kb][16][kb] bytes, so the 16 rows x kb columns of
// one (row tile, k block) are one contiguous block and consecutive blocks of a tile are adjacent; a
// 16-row tile keeps the byte range it has in the row-major layout. Byte offset of element (r, c) of an
// N x K matrix:
__host__ __device__ inline long long blocked_index(long long r, long long c, long long K, int kb) {
    return ((r >> 4) * (K / kb) + c / kb) * 16LL * kb + (r & 15) * kb + c % kb;
}
constexpr int kWeightBlock = 512;  // k per block of the blocked layout

struct GemvParams {
    const void* w;         // [N, K] row-major weights (or blocked, see kb)
    const void* scales;    // int8: f16 [N, K / group]
    int group;             // int8 scale group; >= K means one scale per output row
    int N, K, M;           // W rows, inner dim, activation rows
    const void* x;         // activations [M, K] (x_dtype), row stride x_ld
    int x_dtype;
    long long x_ld;
    const float* norm_w;   // fused RMSNorm of x rows before use (null = off)
    float eps;
    int epi;
    int out_dtype;
    int nseg;
    GemvSeg seg[4];
    unsigned long long* argmax;  // [M] keys for EPI_ARGMAX
    int argmax_base;             // index of W's row 0 in the argmax (vocab shard offset under TP)
    int kt;                      // K elements per shared-memory tile (a multiple of 512)
    int prefetch;                // prefetch the first row block of weights into L2 before pdl_wait
    // Split-K scratch of the one-row bulk GEMV over blocked weights (null: no split): part >= 64 floats
    // (two parts of 16 doubles) per 16-row tile, counters >= one per tile, zero at rest (every launch
    // leaves them zero).
    float* part;
    unsigned* counters;
    int counter_count;
    int kb;      // > 0: int8 W in the blocked layout with this k per block (N % 16 == 0, K % kb == 0)
    int ugroup;  // bulk GEMV: k blocks per unit (set by the dispatcher)
    const PeerSum* peer;  // EPI_PEER_SUM: the communicator's mailboxes (device memory)
    // K-split one-row GEMV over blocked int8 weights: int64 sums per output row, zero at rest (every
    // launch leaves them zero), acc_count >= N; the tile-group counters are `counters`.
    long long* acc;
    int acc_count;
    // L2 prefetch of up to two read-only regions (the weights of a later projection of the step): the
    // k-split GEMV's producer warps issue cp.async.bulk.prefetch.L2 over them, an even slice per CTA,
    // after their first stages. Only that kernel issues them; null or 0 bytes = none. The regions must
    // lie inside allocations and start 16-byte aligned.
    const void* l2pf[2];
    long long l2pf_bytes[2];
};

// Launches y = x * W^T with the fused options in `p` (fills kt and the grid). `w_dtype` is
// L0B_I8 / L0B_F16 / L0B_BF16 / L0B_F32. Rows of x are processed in groups of up to 8 per pass.
l0b_status gemv_nk_launch(l0b_device* dev, int w_dtype, GemvParams p);

// Process-wide choice between the tensor-core GEMV (default) and the fp32-FMA GEMV for the shapes
// both take; launches already recorded into command lists keep the kernel they were recorded with.
void gemv_set_tensor_cores(bool on);
// Process-wide choice of the bulk-copy kernel for one activation row where it applies (default on);
// launches already recorded keep their kernel.
void gemv_set_bulk(bool on);
void gemv_set_fill_split(int s);
void gemv_set_bulk_short_rows(bool on);
void gemv_set_ksplit(bool on);
void gemv_set_ksplit_stages(int s);
// The bulk GEMV's ring of whole tiles: 0 = at most 120 KB of tiles (default), 2..8 = at most that many,
// 1 = as many as its shared-memory budget holds.
void gemv_set_bulk_stages(int s);
// Megabytes of the gate/up weights the one-row decode step prefetches into L2 ahead of their projection
// (the o_proj GEMV issues them; q/k/v also prefetches o_proj's weights and down the next layer's q/k/v);
// 0 = no prefetch. Process-wide; affects steps recorded afterwards.
int gemv_l2_prefetch_mb();
void gemv_set_l2_prefetch_mb(int mb);
// Process-wide: models created afterwards store their int8 per-row-scaled projections with few row
// tiles in the blocked layout (default on).
bool weight_blocking();
void set_weight_blocking(bool on);

// Whether gemv_nk_launch can run `p` (M rows) with the EPI_PEER_SUM epilogue: 16-bit or per-row int8
// weights on the tensor-core GEMV, one f32 output segment, M x N within a mailbox slot.
bool gemv_peer_sum_applies(int w_dtype, const GemvParams& p);
// Whether gemv_nk_launch runs `p` on the k-split GEMV (blocked int8, one row).
bool gemv_takes_ksplit(int w_dtype, const GemvParams& p, int sm_count);
// The communicator's peer-sum mailboxes (device memory), or null: no peer path, or fused all-reduces
// switched off (l0b_comm_set_fused_allreduce).
const PeerSum* comm_peer_sum(const l0b_comm* c);

// Raw-stream variant (no device handle): immediate launch on `stream`.
l0b_status gemv_nk_launch_stream(cudaStream_t stream, int sm_count, int w_dtype, GemvParams p);

// Reference layout [K, N] (y = x * W): Gemv.Execute/ExecuteRows for f32/f16 weights.
l0b_status gemv_kn_launch(l0b_device* dev, int w_dtype, int m, int n, int k, const float* x, const void* w,
                          float* y);
// f32 C[M,N] = A[M,K] * B[K,N] (Gemm.Execute fallback for N % 4 != 0).
l0b_status gemm_f32_launch(l0b_device* dev, int m, int n, int k, const float* a, const float* b, float* c);

}  // namespace l0b
