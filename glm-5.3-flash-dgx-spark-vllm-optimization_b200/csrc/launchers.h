// Host-side launch interface of the glm53 CUDA kernels (raw pointers + stream; no torch headers, so the .cu
// files compile fast). bindings.cpp wraps these for Python.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

// ---------------------------------------------------------------- small-M GEMM (gemv.cu)
enum GemvMode { GEMV_BF16 = 0, GEMV_F32 = 1, GEMV_F32_ACC = 2, GEMV_SWIGLU = 3 };

struct GemvArgs {
  const __nv_bfloat16* x; int64_t ldx; int64_t bsx;   // activations [batch][M][K] (row stride ldx)
  const void* w; int64_t bsw;                          // weights [batch][N][K] (fp8 bytes or bf16)
  const float* scale; int64_t bss;                     // per-row scale [batch][N] (may be null for bf16)
  void* y; int64_t ldy; int64_t bsy;                   // output [batch][M][ldy]
  int M, N, K, batch;
  int mode;
  float limit;                                         // SwiGLU clamp
  // fused all-gather of the fp32 partial (tensor-parallel row-parallel projections, modes F32 / F32_ACC): every
  // output element is also stored into each rank's receive slot `push_rank` over peer memory, and the last CTA
  // raises this rank's arrival flag on every peer (release); null push_ptrs = no push
  float* const* push_ptrs;                             // [world] receive-buffer base on each rank (this parity)
  unsigned* const* push_flags;                         // [world] arrival flags base on each rank (this parity)
  unsigned* push_done;                                 // local CTA completion counter
  int64_t push_slot;                                   // elements per rank slot
  int push_rank, push_world;
  int* err;                                            // device error word (bounded waits)
  int force_ks, force_cl;                              // split-K kernel shape overrides (0 = chosen by size; force_ks
                                                       // -1 = the bulk-copy kernel, -2 = the split-K kernel
                                                       // with its own shape choice)
};
cudaError_t g53_gemv_fp8(const GemvArgs& p, cudaStream_t st);
cudaError_t g53_gemv_bf16(const GemvArgs& p, cudaStream_t st);
// grouped dynamic conv of the block drafter (dconv.cu): out[t] = sum_k bf16(base[k] + delta[t][k][c / gs]) x[t - k]
// within a draft block of block_size rows, with the eager op chain's bf16 roundings
struct DconvArgs {
  const __nv_bfloat16* x; int64_t ldx;       // [T, H] rows (inner stride 1)
  const __nv_bfloat16* delta;                // [T, taps, G] per-row kernel deltas, G = H / gs (contiguous)
  const __nv_bfloat16* base;                 // [taps, H] static kernel
  __nv_bfloat16* out;                        // [T, H] contiguous
  int T, H, taps, gs, G, block_size;
};
cudaError_t g53_dconv(const DconvArgs& a, cudaStream_t st);

// L2 prefetch of up to four weight ranges (l2_prefetch.cu)
struct L2Ranges {
  const char* ptr[4];
  int64_t bytes[4];
  int count;
};
cudaError_t g53_l2_prefetch(const L2Ranges& r, cudaStream_t st);

// persistent bulk-copy (TMA) streamed variant for large fp8 projections (gemv_bulk.cu)
bool g53_gemv_bulk_ok(const GemvArgs& p);
cudaError_t g53_gemv_bulk(const GemvArgs& p, bool pdl, cudaStream_t st);

// ---------------------------------------------------------------- large-M GEMM (gemm_sm100.cu)
struct GemmArgs {
  const void* a; int64_t lda;          // [M, K] activations (bf16 or e4m3), K-major
  const void* b; int64_t ldb;          // [N, K] weights (bf16 or e4m3), K-major
  const float* a_scale;                // [M] (e4m3 activations) or null
  const float* b_scale;                // [N] or null
  void* y; int64_t ldy;
  int M, N, K, mode, fp8;
  float limit;
  int* err;                            // device error word (bounded waits that ran out)
  int vec;                             // set by the launcher: 16-byte epilogue stores allowed
  // batched GEMM (e.g. per attention head): batch strides in elements of A, B, Y and of b_scale
  int batch;                           // 0 or 1: a single GEMM
  int64_t bsa, bsb, bsy, bss;
  // fused tensor-parallel reduction (fp32 modes): every output row is also stored into slot push_rank of every
  // rank's receive buffer (peer memory); the last CTA releases flag [push_rank] on every rank
  float* const* push_ptrs; unsigned* const* push_flags; unsigned* push_done;
  int64_t push_slot; int push_rank, push_world;
  // all-gather + GEMM: A is [ag_world x ag_rows, K] row-sharded over ranks; shard j at ag_ptrs[j] (host array of
  // device addresses, peer memory for j != rank) with row pitch lda; the producer waits for ag_flags[j] >= ag_target
  int ag_world, ag_rows, ag_rank;
  const int64_t* ag_ptrs;                // host array (tensor maps)
  const int64_t* ag_ptrs_dev;            // the same addresses on the device (staging copies)
  const unsigned* ag_flags; unsigned ag_target;
  __nv_bfloat16* ag_stage;               // local [ag_world * ag_rows, K]: peers' rows, copied once per epoch
  int* ag_ready;                         // local [ag_world * ag_rows / 128]: epoch of each staged row block
};
cudaError_t g53_gemm_sm100(const GemmArgs& p, cudaStream_t st);
cudaError_t g53_e4m3_to_bf16(const uint8_t* w, int64_t n, __nv_bfloat16* out, cudaStream_t st);
cudaError_t g53_quant_rows_e4m3(const __nv_bfloat16* x, int64_t ldx, int R, int K, uint8_t* q, float* scale,
                                cudaStream_t st);

// ---------------------------------------------------------------- MoE (moe.cu)
struct RouteArgs {
  const float* logits;        // [R, E] fp32 router logits
  const float* bias;          // [E]
  int R, E, top_k;
  float scale; int norm;
  int* topk_ids;              // [R, top_k]
  float* topk_w;              // [R, top_k]
  // grouping (sorted by expert, then row-major pair index)
  int* group_count;           // [1]   number of distinct experts U
  int* group_expert;          // [max_groups]
  int* group_offset;          // [max_groups + 1]
  int* pair_token;            // [R*top_k] token row of each sorted pair
  int* pair_expert;           // [R*top_k] expert of each sorted pair
  float* pair_w;              // [R*top_k] routing weight of each sorted pair
  int* pair_of;               // [R*top_k] sorted position of pair (r, k)
  int max_groups;
};
cudaError_t g53_moe_route(const RouteArgs& a, cudaStream_t st);

struct Exl3Args {
  // x rows [T, K] (bf16) for rot_in; the experts' stacked tensors
  const __nv_bfloat16* x; int64_t ldx;
  const int16_t* tr_g; const __half* suh_g; const __half* svh_g;    // gate: trellis [E, K/16, N/16, 64]
  const int16_t* tr_u; const __half* suh_u; const __half* svh_u;    // up
  const int16_t* tr_d; const __half* suh_d; const __half* svh_d;    // down [E, N/16, D/16, 64]
  int K;        // hidden (gate/up input, down output)
  int N;        // local expert width (gate/up output, down input)
  int Dout;     // down output width (== K)
  // routing
  const int* group_count; const int* group_expert; const int* group_offset;
  const int* pair_token; const int* pair_expert; const float* pair_w;
  int max_groups, pairs, top_k;
  float limit;
  // scratch
  __half* xh_g; __half* xh_u;   // [pairs, K] rotated inputs
  __half* xd;                   // [pairs, N] rotated down input
  float* yd;                    // [pairs, Dout] weighted expert outputs
  int decode_layout;            // 1: xh/xd rows in the decode fragment layout (moe.cu dup_word); 0: natural order
  // expert parallelism (ep_moe.cu): device-side pair count for rot_in, and the down epilogue's per-pair output
  // row addresses (peer memory) with the flags released by its last CTA
  const int* pair_count;        // [1] or null
  const int64_t* out_ptrs;      // [pairs] or null: output row of each pair (else yd)
  unsigned* done;               // last-CTA counter (out_ptrs mode)
  const int64_t* push_flags;    // [push_world] flag addresses released after the last CTA
  int push_world;
  int launch_groups;            // > 0: grid rows of the group loop (CTAs stride over the group table)
  // decode: weight ranges the gate/up CTAs prefetch into L2 (64 KB bulk prefetches spread over the grid) while the
  // ALU-bound trellis decode leaves HBM idle; count 0 = none
  L2Ranges pf;
  int64_t n_rows, n_experts;    // bounds-checked build: rows of x, experts of the stacked tensors (0: unknown)
};
cudaError_t g53_exl3_rot_in(const Exl3Args& a, cudaStream_t st);
// ---------------------------------------------------------------- expert parallelism (ep_moe.cu)
struct EpArgs {
  // source side (this step's sorted pairs and the peer buffers of parity p)
  const int* n_pairs;                        // [1]
  const int* pair_token; const int* pair_expert; const float* pair_w;
  const __nv_bfloat16* x; int64_t ldx;
  int K, El, rank, world, cap, recv_cap;
  const int64_t* recv_x; const int64_t* recv_meta; const int64_t* recv_cnt;   // [world] peer addresses
  const int64_t* disp_flags;                 // [world] address of disp_flag[p][rank] on each rank
  const int64_t* comb;                       // [world] address of comb[p] on each rank
  unsigned* done; unsigned* done2;           // local last-CTA counters
  unsigned* epoch;                           // local epoch[p]
  int* err;
  // receiver side (this rank's buffers of parity p)
  const unsigned* my_disp_flags;             // [world]
  const unsigned* my_comb_flags;             // [world]
  const int* my_cnt;                         // [world][El]
  const void* my_meta;                       // int4 [world][cap]
  const float* my_comb;                      // [cap][K]
  int* seg_base; int* seg_cnt; int* seg_src;  // [world*El]
  int* n_recv;
  int* group_count; int* group_expert; int* group_offset;   // [1], [El], [El+1]
  int* rp_token; int* rp_expert; float* rp_w; int64_t* rp_out;   // [recv_cap]
};
cudaError_t g53_ep_dispatch(const EpArgs& a, int max_pairs, cudaStream_t st);
// flags[j] = address of rank j's flag array: raise element [rank] on every rank after this rank's prior writes
cudaError_t g53_signal_peers(const int64_t* flags, int rank, int world, cudaStream_t st);
cudaError_t g53_ep_plan(const EpArgs& a, cudaStream_t st);
cudaError_t g53_ep_combine(const EpArgs& a, const int* pair_of, int R, int top_k, float* out, cudaStream_t st);
cudaError_t g53_exl3_gate_up(const Exl3Args& a, cudaStream_t st);
cudaError_t g53_exl3_down(const Exl3Args& a, cudaStream_t st);
// out[r, :] (+)= sum_k yd[pair_of[r, k], :]  (slot order), fp32
cudaError_t g53_moe_combine(const float* yd, const int* pair_of, int R, int top_k, int D, float* out,
                            int accumulate, cudaStream_t st);
// prefill: tcgen05 grouped expert GEMM with in-shared-memory trellis decode (moe_prefill_sm100.cu)
struct MoePrefillArgs {
  const int16_t* tr0; const int16_t* tr1;         // gate/up trellis (gate_up) or down trellis (tr1 unused)
  const __half* svh0; const __half* svh1;         // output scales of tr0 / tr1
  const __half* suh_next;                         // gate_up: suh of the down projection
  const float* pair_w;                            // down: routing weight per sorted pair
  const int* group_count; const int* group_expert; const int* group_offset;
  const __half* x0; const __half* x1;             // rotated inputs [rows, K] (gate, up) or xd (down)
  int64_t rows;                                   // rows of x0 / x1 (sorted pairs)
  int K, N, max_groups;
  void* out;                                      // gate_up: f16 [rows, N] down input; down: f32 [rows, N]
  float limit;
  int* err;
  // expert parallelism (down): per-row output addresses (peer memory) and the flags released by the last CTA
  const int64_t* out_ptrs; unsigned* done; const int64_t* push_flags; int push_world;
  int64_t n_experts;                              // bounds-checked build: experts of the trellis tensors (0: unknown)
};
cudaError_t g53_moe_prefill(const MoePrefillArgs& p, bool gate_up, cudaStream_t st);
// scalable routing for prefill: per-row top-k, expert histogram, scan, scatter (positions within an expert in
// arrival order: outputs per pair do not depend on it)
cudaError_t g53_moe_route_large(const RouteArgs& a, int* counts, int* fill, cudaStream_t st);

// one-tile decode for tests: W_q [K, N] fp16 from trellis [K/16, N/16, 64]
cudaError_t g53_exl3_unpack(const int16_t* tr, int K, int N, __half* out, cudaStream_t st);

// ---------------------------------------------------------------- mHC / norms (mhc.cu)
struct HcArgs {
  __nv_bfloat16* X;           // [R, S, D] residual streams (bf16), updated in place by post
  const float* branch;        // [R, D] fp32 branch output (post) or null (pre only)
  const float* post; const float* comb;   // [R, S], [R, S, S] from the previous pre
  const __nv_bfloat16* fn;    // [n_mix, S*D]
  const float* base; const float* hscale; // [n_mix], [3]
  const __nv_bfloat16* norm_w;  // [D]
  __nv_bfloat16* normed;      // [R, D] out
  float* post_out; float* comb_out;       // [R, S], [R, S, S] out
  float* part;                // [R, NB, 32] scratch partial dots (+ sum of squares in slot n_mix)
  int R, S, D;
  float eps, hc_eps; int iters;
  // fused reduce of the tensor-parallel partials: branch = sum over ranks (rank order) of gath[j] once every rank's
  // arrival flag reached epoch + 1 (bounded wait); null gath = branch is already reduced
  const float* gath;          // [world][slot] receive buffer of this parity (local)
  int64_t gath_slot;
  int world;
  const unsigned* flags;      // [world] arrival flags of this parity (local)
  unsigned* epoch;            // consumptions of this parity so far (local)
  unsigned* done;             // CTA completion counter (local)
  int* err;
  int use_tc;                 // 1: prefill-sized launches (R >= 256, S = 4, no fused reduce) use the tensor cores
  int nb;                     // column blocks of `part` (set by the launcher)
};
cudaError_t g53_hc_post_pre(const HcArgs& a, cudaStream_t st);   // (optional post) then pre
// decode windows (R <= 16, with pre): the whole post + pre in one cluster kernel (mhc_decode.cu)
bool g53_hc_decode_ok(const HcArgs& a);
cudaError_t g53_hc_decode(const HcArgs& a, cudaStream_t st);
// tensor-core partial pass only (post + mixing dots + sums of squares into part [R, D / 512, 32])
cudaError_t g53_hc_partial_tc(const HcArgs& a, cudaStream_t st);
cudaError_t g53_embed(const int* ids, const __nv_bfloat16* table, int V, int R, int D, int S, __nv_bfloat16* X,
                      cudaStream_t st);
cudaError_t g53_stream_mean_norm(const __nv_bfloat16* X, int R, int S, int D, const __nv_bfloat16* w, float eps,
                                 __nv_bfloat16* hidden, __nv_bfloat16* normed, cudaStream_t st);
cudaError_t g53_rmsnorm(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* w, int R, int D, float eps,
                        __nv_bfloat16* y, int64_t ldy, cudaStream_t st);

cudaError_t g53_rmsnorm_f32(const float* x, const __nv_bfloat16* w, int R, int D, float eps, __nv_bfloat16* y,
                            cudaStream_t st);
cudaError_t g53_block_attn(const __nv_bfloat16* qkv, int R, int H, int Dh, int block, float scale, __nv_bfloat16* o,
                           cudaStream_t st);

// ---------------------------------------------------------------- KDA (kda.cu)
struct KdaArgs {
  const __nv_bfloat16* proj; int64_t ldp;   // [R, ldp]: q|k|v (3*H*Dh) then f_a, g_a, b (H) at b_off
  const __nv_bfloat16* f;                    // [R, H*Dh] f_b output (decay logits)
  const __nv_bfloat16* gate;                 // [R, H*Dh] g_b output (output gate logits)
  const float* conv_w;                       // [3*H*Dh, taps]
  __nv_bfloat16* conv_pool;                  // [slots][taps-1][3*H*Dh] conv windows (rows oldest first)
  const float* a_log; const float* dt_bias;  // [H], [H*Dh]
  const __nv_bfloat16* o_norm;               // [Dh]
  float* S_pool;                             // [states][H][Dh][Dh] recurrent states (v-major)
  __nv_bfloat16* qkv;                        // [R, 3*H*Dh] conv outputs (kept for replay)
  float* o_raw;                              // [R, H*Dh] recurrent outputs before the gated norm (may be null)
  __nv_bfloat16* out;                        // [R, H*Dh] gated-normed output
  // sequences of the launch: rows [row0[b], row0[b] + nrows[b])
  const int* row0; const int* nrows;         // [B]
  const int* s_in; const int* s_out;         // [B] state pool index read / written
  const int* conv_slot;                      // [B] conv pool slot
  int B, max_rows;                           // sequences, max rows of one sequence
  int R, H, Dh, taps, b_off;
  float lower, eps;
  float* scr; int scr_slots;                 // chunked prefill: per-(chunk slot, head) records (kda_chunk.cu)
  // fused decode step (kda_decode.cu): the f_b / g_b projections of the f_a / g_a columns computed in the kernel
  const uint8_t* fb_w; const float* fb_s;    // [H*Dh, Dh] e4m3, [H*Dh] row scales
  const uint8_t* gb_w; const float* gb_s;
  int fa_off;                                // column of f_a in proj (g_a follows at fa_off + Dh)
  __nv_bfloat16* f_store;                    // [R, H*Dh] decay logits kept for the commit replay
  int64_t n_states, n_conv;                  // bounds-checked build: state-pool and conv-pool slots (0: unknown)
};
cudaError_t g53_kda_conv(const KdaArgs& a, cudaStream_t st);          // qkv = silu(conv(window ++ proj rows))
cudaError_t g53_kda_recurrent(const KdaArgs& a, cudaStream_t st);     // per sequence: S_in -> S_out, o_raw
cudaError_t g53_kda_gated_norm(const KdaArgs& a, cudaStream_t st);    // out = rmsnorm(o_raw) * w * sigmoid(gate)
cudaError_t g53_kda_conv_commit(const KdaArgs& a, cudaStream_t st);   // window <- last taps-1 of window ++ nrows rows
// one kernel for a decode window: f_b, g_b, conv, recurrence and gated norm (kda_decode.cu)
bool g53_kda_decode_ok(const KdaArgs& a);
cudaError_t g53_kda_decode(const KdaArgs& a, cudaStream_t st);
// chunked (64-token) form of g53_kda_recurrent for prefill: same inputs/outputs, per-sequence rows in chunks;
// needs a.scr with g53_kda_chunk_scratch_floats(max_rows, max_seqs, H, Dh) floats (scr_slots = rows/64 + seqs + 1)
cudaError_t g53_kda_chunk(const KdaArgs& a, cudaStream_t st);
int64_t g53_kda_chunk_scratch_floats(int max_rows, int max_seqs, int H, int Dh);

// ---------------------------------------------------------------- MLA / DSA (mla.cu, dsa.cu)
struct MlaPrepArgs {
  const __nv_bfloat16* qkv_a; int64_t ld;    // [R, q_lora + kv_lora + rope]
  const __nv_bfloat16* q_norm; const __nv_bfloat16* kv_norm;
  __nv_bfloat16* qr;                          // [R, q_lora]
  uint8_t* kv_cache; float* kv_scale; __nv_bfloat16* kpe_cache;   // latent cache (per slot)
  const int* slots;                           // [R] cache slot of each row
  const int* positions;                       // [R] absolute positions (rope)
  int R, q_lora, kv_lora, rope;
  float eps, theta;
  int64_t n_slots;                            // bounds-checked build: cache slots (0: unknown)
};
cudaError_t g53_mla_prep(const MlaPrepArgs& a, cudaStream_t st);
cudaError_t g53_rope_q(__nv_bfloat16* q, int R, int H, int qk, int nope, int rope, const int* positions, float theta,
                       cudaStream_t st);

struct MlaAttnArgs {
  const __nv_bfloat16* q_lat;   // [R, H, L] absorbed queries (bf16)
  const __nv_bfloat16* q_pe;    // rope part of the queries: row r head h at q_pe + r*q_pe_ld + h*q_pe_hs (or null)
  int64_t q_pe_ld; int q_pe_hs;
  const uint8_t* kv_cache; const float* kv_scale; const __nv_bfloat16* kpe_cache;
  const int* sel;               // [R, max_sel] selected cache slots
  const int* sel_count;         // [R]
  int max_sel;
  int R, H, L, rope;
  float sm_scale;
  int splits;                   // key splits (flash-decoding); chunk = ceil(max_sel / splits)
  float* part_o;                // [R, splits, H, L] scratch
  float* part_ml;               // [R, splits, H, 2]
  __nv_bfloat16* o_lat;         // [R, H, L] out (bf16)
  int use_tc;                   // 1: tensor-core kernel (L = 512, no rope, H <= 64); 0: CUDA-core kernel
  int* err;                     // error word of the bounded waits (tensor-core kernel)
  int64_t n_slots;              // bounds-checked build: cache slots (0: unknown)
};
cudaError_t g53_mla_decode(const MlaAttnArgs& a, cudaStream_t st);
// tensor-core attention only (no merge); splits > 1 leaves partials in part_o / part_ml
cudaError_t g53_mla_attn_tc(const MlaAttnArgs& a, cudaStream_t st);

constexpr int kDsaRing = 32;     // tail-ring positions per sequence (>= a window's rows + kpool - 1)
struct DsaArgs {
  const float* iproj; int64_t ldi;  // [R, ID + IH + ID] fp32: index key | head weights | pool gate scores
  const float* ln_w; const float* ln_b; const float* ape;   // [ID], [ID], [kpool, ID]
  const __nv_bfloat16* qi;       // [R, IH*ID] index queries (bf16, before the Hadamard transform)
  // raw index keys and pool gate scores are kept only until their pool is complete: this launch's rows in row
  // buffers, earlier tokens of a still-open pool in a per-sequence tail ring of kDsaRing positions
  __nv_bfloat16* ik_cache;       // [rows, ID] normalised index keys of this launch's rows (bf16)
  float* ig_cache;               // [rows, ID] pool gate scores of this launch's rows
  __nv_bfloat16* ik_ring;        // [state slots * kDsaRing, ID] tail ring of index keys
  float* ig_ring;                // [state slots * kDsaRing, ID] tail ring of gate scores
  const int* seq_desc; int seq_ld;   // [5, sequences]: row0, nrows, s_in, s_out, state slot (the ring owner)
  uint8_t* pool_cache; float* pool_scale;   // [pool slots, ID] e4m3, [pool slots] power-of-two scales
  const int* slots;              // [R] token slot of each row
  const int* positions;          // [R] absolute position of each row
  const int* block_table;        // token page tables [sequences, max_blocks]
  const int* row_seq;            // [R] sequence (page-table row) of each row
  int bt_ld;
  int block_size;                // tokens per page (a multiple of kpool)
  int R, IH, ID, kpool, topk_pools;
  float eps;
  float* logits;                 // [R, max_pools] scratch
  int max_pools;
  int* sel; int* sel_count; int max_sel;   // out: selected token slots per row
  int* err;                      // device error word (bounded waits of the tensor-core logits kernel)
  int64_t n_pools;               // bounds-checked build: pool slots of the index cache (0: unknown)
  int64_t n_owners;              // bounds-checked build: ring owners (state slots) of the tail rings (0: unknown)
  // decode windows launch both logits kernels; each runs only on its side of this pool count (the longest row of
  // the launch decides): CUDA cores up to it, tcgen05 above it.  0: the kernel runs unconditionally.
  int tc_min_pools;
};
#ifdef __CUDACC__
// true when the longest row of the launch has more complete pools than a.tc_min_pools (every warp forms the same
// answer from the same positions)
__device__ __forceinline__ bool dsa_long_rows(const DsaArgs& a) {
  int mx = 0;
  for (int r = threadIdx.x & 31; r < a.R; r += 32) mx = max(mx, a.positions[r] / a.kpool);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  return mx > a.tc_min_pools;
}
#endif
cudaError_t g53_dsa_update(const DsaArgs& a, cudaStream_t st);   // index keys, gate scores, completed pools
cudaError_t g53_dsa_logits(const DsaArgs& a, cudaStream_t st);  // pool logits of every row (CUDA cores)
cudaError_t g53_dsa_logits_tc(const DsaArgs& a, cudaStream_t st);   // same on tcgen05 (dsa_tc.cu)
cudaError_t g53_dsa_select(const DsaArgs& a, cudaStream_t st);

// ---------------------------------------------------------------- sampling / verify (sample.cu)
cudaError_t g53_argmax_rows(const float* logits, int R, int V, int64_t ld, int vocab_offset, float* best_val,
                            int* best_id, cudaStream_t st);
struct VerifyArgs {
  const int* draft;          // [B, K] draft tokens
  const int* target_argmax;  // [B, K+1] target greedy tokens per verify row
  int B, K;
  int forced;                // accept all K drafts (benchmark mode)
  int* accepted;             // [B] accepted draft count
  int* next_tokens;          // [B, K+1] emitted tokens (accepted drafts + correction/bonus)
};
cudaError_t g53_greedy_verify(const VerifyArgs& a, cudaStream_t st);
struct RejectArgs {
  const float* target_probs;   // [B, K+1, V]
  const float* draft_probs;    // [B, K, V]
  const int* draft;            // [B, K]
  int B, K, V;
  uint64_t seed; const int64_t* positions;   // [B] position of row 0
  int block;                   // 0: standard rejection, 1: block verification
  int* accepted; int* next_tokens;
  float* scratch;              // [B, K+1] block acceptance stats
};
cudaError_t g53_rejection_sample(const RejectArgs& a, cudaStream_t st);
