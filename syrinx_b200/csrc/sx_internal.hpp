// sx_internal.hpp — device data layout and kernel launch interfaces of the B200 path.
//
// HBM layout (all device memory owned by the library):
//   Q8_0 weight [N][K]  -> tile records: ceil(N/16) tiles of 16 rows, each stored as K/32
//                          consecutive 544-byte records, one per 32-wide k block:
//                            [0, 512)   the 16 x 32 int8 quants in the A-operand fragment
//                                       order of mma.m16n8k32 (row-major A): lane t = 4g + c
//                                       owns bytes [16t, 16t + 16) = {row g, k 4c..4c+3 |
//                                       row g+8, same k | row g, k 16+4c.. | row g+8, k 16+4c..}
//                            [512, 544) the 16 f16 block scales as 8 words {d[w], d[w+8]}
//                          so one coalesced 16-byte load per lane feeds one tensor-core
//                          instruction and a matrix is one contiguous stream of exactly
//                          N x K x 34/32 bytes. Rows past N are zero. w1/w3 are interleaved
//                          per tile: tile j holds gate rows 8j..8j+7 then up rows 8j..8j+7.
//   Q4_K weight [N][K]  -> q : u8   [N][K/2] (GGML nibble order inside each 256 super-block)
//                          meta : 16 B [N][K/256] = {f16 d, f16 dmin, u8 scales[12]}
//                          w1/w3 interleaved row by row (g0,u0,g1,u1,...).
//   F32  weight [N][K]  -> f : f32 [N][K] (w1/w3 interleaved row by row)
//   The GGML array-of-blocks layouts are rewritten into these forms at load, losslessly.
//   KV cache: f32 (default) or bf16 pages of PAGE positions, per layer
//   [2][n_pages][Hkv][PAGE][hd], with a per-sequence page table [max_batch][pages_per_seq]
//   of int32 page ids.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/syrinx_dualar.h"

namespace sx {

constexpr int kPage = 64;         // KV positions per page
constexpr int kMaxTok = 8;        // max sequences of a batched decode step
constexpr int kMaxPrefillTok = 64;  // tokens per prefill chunk (max tokens per GEMV launch)
constexpr int kAttnThreads = 256;  // 8 warps per attention CTA
constexpr int kMaxCluster = 8;     // max splits of the attention key axis (one portable cluster)
constexpr int kMaxGroup = 8;      // max query heads per kv head handled in one CTA
constexpr int kQkvChunks = 16;    // max wqkv k-chunks the decode attention adds itself (dim <= 4096)
constexpr int kMaxStops = 256;    // stop ids; more than 4 only right next to the semantic range

// The stop ids [stop_token_id, +num_stop_tokens) continue the semantic range (or end right
// before it), so one widened row range covers both.
inline bool stops_adjacent(const sx_model_desc& d) {
  const uint64_t t0 = d.stop_token_id, t1 = t0 + (uint32_t)d.num_stop_tokens;
  return t0 == (uint64_t)d.semantic_end_id + 1 || t1 == d.semantic_begin_id;
}

struct DevMat {
  int dtype = -1;
  int64_t rows = 0, cols = 0;
  void* q = nullptr;        // Q8_0 tile records / Q4_K nibbles / F32 values
  uint8_t* meta = nullptr;  // Q4_K 16-B super-block headers
  size_t bytes() const;
};

// Q4_K layer matrices as tile records for the integer tensor-core GEMV (the loader's internal
// dtype; emb / head tables keep the row layout). One record = 16 rows x one 256-wide
// super-block, kQ4Rec bytes:
//   [0, 2048)     quants: 4 pairs of 32-wide sub-blocks x 512 B; lane L = 4g + c owns 16 bytes
//                 of each pair: for sub-block 2jp + h, bytes 8h..8h+3 hold row g and 8h+4..8h+7
//                 row g + 8, byte i = q[k = 4c + i] | q[k = 16 + 4c + i] << 4 (nibbles 0..15),
//                 so `& 0x0F0F0F0F` and `>> 4 & ...` give the mma.m16n8k32 A fragment words;
//   [2048, 2176)  6-bit sub-block scales: per g, 8 bytes of row g then 8 bytes of row g + 8;
//   [2176, 2304)  6-bit sub-block mins, the same order;
//   [2304, 2368)  per g: f16 d and dmin of row g, then of row g + 8.
// 2368 bytes per 4096 weights (GGML: 2304).
constexpr int kDtypeQ4KT = 64;
constexpr int kQ4Rec = 2368;
__host__ __device__ inline int q4_quant_off(int rr, int j, int k) {  // byte of (tile row, sub-block, k); nibble k >> 4
  const int g = rr & 7, c = (k & 15) >> 2;
  return (j >> 1) * 512 + (4 * g + c) * 16 + (j & 1) * 8 + (rr >> 3) * 4 + (k & 3);
}
__host__ __device__ inline int q4_sc_off(int rr, int j) { return 2048 + (rr & 7) * 16 + (rr >> 3) * 8 + j; }
__host__ __device__ inline int q4_dd_off(int rr) { return 2304 + (rr & 7) * 8 + (rr >> 3) * 4; }

// Q8_0 tile-record geometry (see the layout above).
constexpr int kQ8Tile = 16;
constexpr int kQ8Rec = 544;
inline int64_t q8_tiles(int64_t rows) { return (rows + kQ8Tile - 1) / kQ8Tile; }
// byte offset of quant (tile row rr, k kk) inside its record
__host__ __device__ inline int q8_quant_off(int rr, int kk) {
  return ((rr & 7) * 4 + ((kk & 15) >> 2)) * 16 + ((kk >> 4) * 2 + (rr >> 3)) * 4 + (kk & 3);
}
// byte offset of tile row rr's f16 scale inside its record
__host__ __device__ inline int q8_scale_off(int rr) { return 512 + (rr & 7) * 4 + (rr >> 3) * 2; }

struct DevLayer {
  float* attn_norm = nullptr;
  float* bqkv = nullptr;
  float* qn = nullptr;
  float* kn = nullptr;
  float* bo = nullptr;
  float* ffn_norm = nullptr;
  DevMat wqkv, wo, w13, w2;
};

// ---- kernel argument bundles --------------------------------------------------------

enum Epi : int {
  EPI_STORE = 0,   // y[m][row] = acc (+ bias[row])
  EPI_ADD = 1,     // y[m][row] = y[m][row] + (acc (+ bias[row]))   (residual add)
  EPI_SWIGLU = 2,  // y[m][j] = silu(gate_j) * up_j, pairs as the w1/w3 interleave places them
  EPI_ARGMAX = 3,  // logits (stored if y != null) + packed argmax over allowed rows
  EPI_NONE = 4,    // Q8_0 / Q4_K records only: partials, no merge launch; the consumer adds
                   // the k-chunks itself (decode attention reading the wqkv partials, the
                   // one-token w2 GEMV reading the w1|w3 partials)
};

// Tensor parallelism: one process per GPU; the wo / w2 residual merges exchange per-rank
// partial rows over NVLink (peer pointers from CUDA IPC) instead of an all-reduce call.
// Every rank owns a receive region rx[2 parities][kMaxTp source ranks][xb_cap] of 8-byte
// words {f32 value | u32 exchange epoch << 32}; senders store straight into the peers'
// regions, receivers poll their own words until the epoch matches. The epoch of a slot
// (token m, row) counts the exchanges that carried that slot, identically on every rank.
constexpr int kMaxTp = 8;  // ranks in a tensor-parallel group
struct TpComm {
  int rank = 0, size = 1;             // size 1: no tensor parallelism
  uint64_t* rx[kMaxTp] = {};          // each rank's receive region as mapped on this GPU
  uint32_t* slot_epochs = nullptr;    // this rank's per-slot exchange counters [xb_cap]
  int* err = nullptr;                 // this rank's device error flag (3: a peer did not arrive)
  int xb_cap = 0;                     // slots (tokens x rows) per (parity, source rank)
  uint64_t wait_ns = 5000000000ull;   // longest wait for a peer's word (%globaltimer ns)
};

struct GemvArgs {
  DevMat w;
  const float* x = nullptr;  // [M][K] activations (row stride K)
  const float* norm_w = nullptr;  // non-null: RMSNorm prologue with this gain over K
  float eps = 0.f;
  const float* bias = nullptr;  // [N] f32
  float* y = nullptr;           // output (row stride ldy)
  int ldy = 0;
  int M = 1;
  // logical -> physical row map (head over a row subset): i < n_range -> row_base + i,
  // else extra[i - n_range]
  int row_base = 0, n_range = 0, n_extra = 0;
  int extra[4] = {0, 0, 0, 0};
  // argmax epilogue: allowed = [allow_lo, allow_hi] U [stop_lo, stop_hi) (stops when !mask)
  unsigned long long* amax = nullptr;  // [M] packed (orderable f32 << 32 | ~row)
  uint32_t allow_lo = 0, allow_hi = 0, stop_lo = 0, stop_hi = 0;
  // Q8_0 only: per-(tile, k-chunk) partial sums, part_cap floats (q8_part_floats)
  float* part = nullptr;
  size_t part_cap = 0;
  // residual add across a tensor-parallel group (EPI_ADD of a K-split matrix, Q8_0 only)
  TpComm tp;
  // One token, Q8_0, no RMSNorm: x is not read; x[j] = silu(gate_j) * up_j is formed from the
  // w1|w3 GEMV's partials [tile][glu_nc][1][16] (left by EPI_NONE), added in k_merge_q8's order
  const float* glu_part = nullptr;
  int glu_nc = 0;
  int* err = nullptr;  // device error flag (bounded pipeline waits of the tensor-core GEMM)
  uint8_t* tc_scratch = nullptr;  // the tensor-core GEMM's B operands (gemm_tc_scratch_bytes)
  size_t tc_scratch_bytes = 0;
};
// floats of partial sums a Q8_0 GEMV over `w` with `n_rows` logical rows needs at M tokens
size_t q8_part_floats(const DevMat& w, int64_t n_rows, int M);

struct AttnArgs {
  const float* qkv = nullptr;  // [M][(H + 2 Hkv) hd]
  float* out = nullptr;        // [M][H hd]
  void* kbase = nullptr;       // this layer's K pages (f32 or bf16 elements)
  void* vbase = nullptr;       // this layer's V pages
  int kv_f32 = 1;              // element type of the cache: 1 f32, 0 bf16
  const int* page_table = nullptr;  // [batch][pt_stride]
  int pt_stride = 0;
  const int* tok_seq = nullptr;  // [M] sequence of each token
  const int* tok_pos = nullptr;  // [M] absolute position of each token (null: const_pos)
  int const_pos = 0;
  const float* qn = nullptr;
  const float* kn = nullptr;
  float eps = 0.f;
  const float* inv_freq = nullptr;
  int interleaved = 1;
  float scale = 1.f;  // f32(1/sqrt(hd)) computed in double on the host (s2/nn.rs:344)
  int H = 0, Hkv = 0, hd = 0;
  int n_split = 1;  // splits of the key axis = cluster size (<= kMaxCluster)
  int append = 1;  // 1: this launch appends each token's own K/V (decode)
  int M = 1;
  // Decode: when non-null, q|k|v come from the wqkv GEMV's k-chunk partials
  // [tile][qkv_nc][qkv_mt][16] (EPI_NONE), added here in k_merge_q8's order, plus qkv_bias,
  // instead of from the merged rows in qkv.
  const float* qkv_part = nullptr;
  int qkv_nc = 0;  // k-chunks of the wqkv GEMV (<= kQkvChunks)
  int qkv_mt = 1;  // its template token count (the power of two >= M)
  const float* qkv_bias = nullptr;
};

// ---- launchers (stream-ordered, programmatic dependent launch enabled) ----------------
// launch_gemv: Q8_0 weights run the tensor-core kernel plus its merge (gemv_q8.cu),
// Q4_K / F32 the register-streaming kernel (gemv.cu).
cudaError_t launch_gemv(const GemvArgs& a, Epi epi, cudaStream_t st);
cudaError_t launch_gemv_q8(const GemvArgs& a, Epi epi, cudaStream_t st);
// Q8_0 partials of 9..64 tokens on tcgen05 (gemm_tc.cu); SYRINX_TC=0 keeps them on mma.sync
bool tc_enabled();
size_t gemm_tc_scratch_bytes(int K, int Mt);
cudaError_t launch_gemm_tc(const GemvArgs& a, int Mt, int K, int nb, int nc, int t_first, int n_vt, int sms,
                           cudaStream_t st);
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st);
cudaError_t launch_kv_append(const AttnArgs& a, cudaStream_t st);
cudaError_t launch_attention_prefill(const AttnArgs& a, cudaStream_t st);

// ---- persistent decode stack (stack.cu) ------------------------------------------------
// One layer's Q8_0 tile records and vectors, as the persistent kernel reads them (device array).
struct StackLayer {
  const uint8_t* wqkv = nullptr;
  const uint8_t* wo = nullptr;
  const uint8_t* w13 = nullptr;
  const uint8_t* w2 = nullptr;
  const float* attn_norm = nullptr;
  const float* bqkv = nullptr;
  const float* qn = nullptr;
  const float* kn = nullptr;
  const float* bo = nullptr;
  const float* ffn_norm = nullptr;
};
constexpr int kStackChunkBlocks = 16;  // 32-wide k blocks per weight item of the persistent stack
struct StackGeo {
  int K = 0, nb = 0, nc = 0, n_vt = 0;  // columns, 32-wide blocks, 16-block k chunks, 16-row tiles
};
struct StackArgs {
  const StackLayer* layers = nullptr;  // device [n_layer]
  int n_layer = 0;
  int dim = 0, H = 0, Hkv = 0, hd = 0, F = 0;
  float eps = 0.f;
  const float* inv_freq = nullptr;
  int interleaved = 1;
  float scale = 1.f;
  uint8_t* kv = nullptr;  // layer l's K pages at kv + l * kv_layer_elems * elem, V half after
  size_t kv_layer_elems = 0;
  int kv_f32 = 1;
  const int* page_table = nullptr;
  int pt_stride = 0;
  const int* tok_seq = nullptr;
  const int* tok_pos = nullptr;  // null: every token at const_pos
  int const_pos = 0;
  int M = 1;        // tokens (1..8)
  int n_split = 1;  // splits of the key axis per (token, kv head)
  float* x = nullptr;   // [M][dim] residual stream, updated in place
  float* xb = nullptr;  // [M][dim] scratch
  float* part0 = nullptr;  // GEMV partials [M][rows][k chunks padded to 4], two alternating buffers
  float* part1 = nullptr;
  float* attn_part = nullptr;  // [M][H][hd][splits] + [M][H][2][splits], splits padded to 4
  float* ss = nullptr;         // sums of squares per k chunk [2][8][64]
  unsigned long long* bar = nullptr;  // grid barrier counter (monotonic)
  int* err = nullptr;
  StackGeo geo[4];  // wqkv, wo, w1|w3, w2
  int nc_dim = 0;   // k chunks of dim
  int nslot = 0;    // ring slots (set by the launcher)
  int inflight = 0;  // weight items the producer keeps in flight (0: the default)
  int l2_ahead = 0;  // items the producer's L2 prefetch cursor may run ahead of the ring (0: off)
  // profiling: non-null -> per CTA [n_layer * 15 + 3] %globaltimer stamps (start; per layer
  // and phase: phase start, prologue end, arrival; final phase start; end)
  unsigned long long* trace = nullptr;
};
bool stack_supported(const StackArgs& a, int sms);
size_t stack_attn_part_floats(int max_tok, int H, int hd);
size_t stack_part_floats(const StackGeo& g, int M);
int stack_max_splits(int sms, int M, int Hkv);
cudaError_t launch_stack(const StackArgs& a, int sms, cudaStream_t st);

struct EmbedArgs {
  const int* tok_seq = nullptr;
  const uint32_t* frames = nullptr;  // [batch][1+C] per-sequence current frame
  int frame_stride = 0;
  const uint32_t* ids = nullptr;  // prompt ids [(1+C) x T] when frames == null
  int T = 0, t0 = 0;               // column offset into the prompt
  DevMat emb, cb_emb;
  int dim = 0, C = 0, R = 0, vocab = 0;
  uint32_t sem_lo = 0, sem_hi = 0;
  int scale_cb = 0;
  float* h = nullptr;  // [M][dim]
  int M = 1;
  int* err = nullptr;  // device error flag (id out of range)
};
cudaError_t launch_embed(const EmbedArgs& a, cudaStream_t st);

// fast-AR / frame bookkeeping kernels (greedy device loop)
struct FrameArgs {
  int M = 1;
  const int* tok_seq = nullptr;
  unsigned long long* amax = nullptr;  // [M] packed argmax (null: code already in the frame)
  uint32_t* frames = nullptr;          // [batch][1+C] current frame per sequence
  int frame_stride = 0;
  int slot = 0;                        // frame column written (0 semantic, 1+c code c)
  uint32_t sem_begin = 0;
  int R = 0;
  DevMat emb;          // fast_embeddings (next fast input) — optional
  float* x = nullptr;  // [M][dim] next fast input
  int dim = 0;
  const float* h_last = nullptr;  // slow residual (for the fast prefix)
  const float* norm_w = nullptr;  // final norm gain (post-norm hidden) or null (pre-norm)
  float eps = 0.f;
  int write_first_code = 0;
  int* done = nullptr;            // [batch] stop flags
  uint32_t stop_lo = 0, stop_hi = 0;
};
cudaError_t launch_take_semantic(const FrameArgs& a, cudaStream_t st);
cudaError_t launch_take_code(const FrameArgs& a, cudaStream_t st);
cudaError_t launch_final_norm(const float* h, const float* w, float eps, int dim, int M, float* out,
                              cudaStream_t st);

struct AdvanceArgs {
  int M = 1;
  const int* tok_seq = nullptr;
  int* tok_pos = nullptr;
  int* seq_len = nullptr;
  const int* done = nullptr;
  const uint32_t* frames = nullptr;
  int frame_stride = 0;
  uint32_t* ring = nullptr;  // [max_frames][batch][1+C]
  int ring_frames = 0;
  int* frame_count = nullptr;  // [batch]
  int batch = 0;
};
cudaError_t launch_advance(const AdvanceArgs& a, cudaStream_t st);

// repack / dequant
// destination row of source row r is r * row_mul + row_add (w1/w3 interleave); for Q8_0
// it is (r / grp) * grp * row_mul + row_add * grp + r % grp (grp 8: the per-tile interleave)
cudaError_t repack_q8_0(const uint8_t* blocks, int64_t rows, int64_t cols, uint8_t* rec, int row_mul, int row_add,
                        int grp, cudaStream_t st);
cudaError_t repack_q4k_tiles(const uint8_t* blocks, int64_t rows, int64_t cols, uint8_t* rec, int row_mul,
                             int row_add, int grp, cudaStream_t st);
cudaError_t repack_q4_k(const uint8_t* blocks, int64_t rows, int64_t cols, uint8_t* q, uint8_t* meta,
                        int row_mul, int row_add, cudaStream_t st);
cudaError_t dequant_blocks(int dtype, const uint8_t* blocks, int64_t n_blocks, float* out,
                           cudaStream_t st);
// sx_dequantize through static device scratch (noalloc.cu): returns an SX_* status
int dequantize_noalloc(int32_t dtype, const void* blocks, int64_t n_blocks, float* out, int32_t device);

// device sampler (sample_dev.cu): the reference Sampler for one sequence, one CTA per draw
constexpr int kSampleMaxIds = 7168;  // allowed ids per draw (shared memory: 216 KB at the cap)
constexpr int kMaxRasWin = 64;       // longest RAS window the device keeps
struct SampleState {                 // per sequence, in device memory
  unsigned long long rng;            // SplitMix64 state
  int win_count;                     // semantic ids pushed so far
  uint32_t win[kMaxRasWin];          // ring of the last ras_win_size of them
};
struct SampleArgs {
  const float* logits = nullptr;          // indexed by vocabulary id (allowed rows written)
  int ranges = 1;                         // allowed ids [lo[j], hi[j]), ascending, disjoint
  uint32_t lo[2] = {0, 0}, hi[2] = {0, 0};
  const sx_sampling_params* params = nullptr;  // device copy
  int semantic = 0;                       // 1: sample_semantic (normal + RAS high draw)
  uint32_t sem_lo = 0, sem_hi = 0;        // is_semantic: [sem_lo, sem_hi]
  uint32_t stop_lo = 0, stop_hi = 0;      // stop ids: [stop_lo, stop_hi) (not pushed to the window)
  uint32_t full_last = 0;                 // last id of the reference's full logits array
  SampleState* st = nullptr;
  unsigned long long* amax = nullptr;     // out: packed key of the drawn id
};
cudaError_t launch_sample(const SampleArgs& a, cudaStream_t st);

// host helpers
void set_error(const std::string& msg);
// Programmatic dependent launch is on unless SYRINX_PDL=0 (plain stream ordering).
bool pdl_enabled();
// Launch config with the programmatic-stream-serialization attribute when enabled.
cudaLaunchConfig_t launch_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t st, cudaLaunchAttribute* attr);
int ggml_row_bytes(int dtype, int64_t cols, size_t* out);

}  // namespace sx
