// Raw-pointer launchers of the sm_100a kernels (no framework types).
// dtype codes: AHB_F32 = 0, AHB_BF16 = 1.  All launches go to `st`.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#define AHB_F32 0
#define AHB_BF16 1

// elementwise.cu
void ahb_sanitize(void* out, const void* in, int64_t n, int dtype, float clip, cudaStream_t st);
void ahb_rmsnorm_fwd(const void* x, const float* scale, void* y, float* rstd, int64_t M, int D, int dtype, float eps,
                     cudaStream_t st);
int ahb_rmsnorm_bwd_blocks(int64_t M, int D);
void ahb_rmsnorm_bwd(const void* dy, const void* x, const float* scale, const float* rstd, void* dx, float* dscale_acc,
                     float* dscale_part, int64_t M, int D, int dtype, cudaStream_t st);
void ahb_conv1d_fwd(const void* x, int64_t xs, const void* w, int wdtype, const float* bias, void* y, int B, int L,
                    int C, int dtype, int silu, float clip, cudaStream_t st);
void ahb_conv1d_bwd(const void* x, int64_t xs, const void* w, int wdtype, const float* bias, const void* dy, void* dx,
                    float* dw_acc, float* db_acc, int B, int L, int C, int dtype, int silu, float clip,
                    cudaStream_t st);
void ahb_accumulate(float* acc, const void* g, int64_t n, int dtype, float scale, cudaStream_t st);
// h = silu(a) * b over bf16 (n % 8 == 0, 16-byte aligned) and its backward
void ahb_swiglu_fwd(const void* a, const void* b, void* h, int64_t n, cudaStream_t st);
void ahb_swiglu_bwd(const void* dh, const void* a, const void* b, void* da, void* db, int64_t n, cudaStream_t st);
// out[c] += sum_b part[b * D + c]
void ahb_colsum_add(const float* part, int nb, int D, float* out, cudaStream_t st);
void ahb_embedding_fwd(const int64_t* ids, const void* emb, int edtype, void* out, int odtype, int64_t T, int D,
                       int64_t V, cudaStream_t st);
void ahb_embedding_bwd(const int64_t* ids, const void* dout, int dtype, float* acc, int64_t T, int D, int64_t V,
                       cudaStream_t st);

// GDN-2 (head dim 128, chunk 64; sequence tensors (B, L, H, 128), chunk tensors (B, H, L/64, ...))
// gdn_tc.cu: chunk-local forward and the two state recurrences on tcgen05.  The chunk
// intermediates wt/u/qg/kg (B, H, L/64, 64 x 128) and aqk (B, H, L/64, 64 x 64) are bf16 tile
// images in the 128-byte-swizzled shared-memory layout, as are at_t (A, 64 x 64), h_store /
// dh_store (128 x 128 per chunk) and vn_store / dvn_store (64 x 128 per chunk).
// Return 0, or a negative code when a launch or set-up failed; `err` receives device timeouts.
int ahb_gdn_chunk_fwd_tc(const void* q, const void* k, const void* v, const float* g, const void* bg, const void* wg,
                         float scale, int B, int L, int H, void* wt_t, void* u_t, void* qg_t, void* kg_t, void* aqk_t,
                         float* gcl, void* at_t, int* err, cudaStream_t st);
int ahb_gdn_state_fwd_tc(const void* wt_t, const void* u_t, const void* qg_t, const void* kg_t, const void* aqk_t,
                         const float* gcl, float scale, int B, int L, int H, const float* h0, void* o, float* h_final,
                         void* h_store, void* vn_store, int* err, cudaStream_t st);
int ahb_gdn_state_bwd_tc(const void* wt_t, const void* qg_t, const void* kg_t, const void* aqk_t, const float* gcl,
                         const void* dout, float scale, int B, int L, int H, const float* dh_final, void* dh_store,
                         void* dvn_store, float* dh0, int* err, cudaStream_t st);
int ahb_gdn_chunk_bwd_tc(const void* q, const void* k, const void* v, const float* g, const void* bg, const void* wg,
                         const void* dout, const void* hs_t, const void* dhs_t, const void* vn_t, const void* dvn_t,
                         const void* at_t, float scale, int B, int L, int H, void* dq, void* dk, void* dv, void* db,
                         void* dw, float* dg, int* err, cudaStream_t st);

// Mamba2 SSD (head dim 64, d_state 128, chunk 64; x, dt (B,L,H,64); B, C (B,L,128); A (H,) fp32)
// ssd_tc.cu: forward (chunk kernel + state recurrence), the reverse state-gradient recurrence and
// the chunk-parallel backward.
// Per chunk-head scratch: send_t (128 x 64 bf16 image), yd_t (64 x 64 fp32 rows), dec_t (64 x 64
// bf16 image), cl (64 fp32); sin_t / dse_t are per chunk-head 128 x 64 bf16 images (rows s,
// columns p) of the incoming state and of the gradient reaching the chunk's end state.
int ahb_ssd_supported(int P, int N);
int ahb_ssd_fwd_tc(const void* x, const void* dt, const float* A, const void* Bm, const void* Cm, int B, int L, int H,
                   void* send_t, void* yd_t, void* dec_t, float* cl, const float* s0, float* s_final, void* y,
                   void* sin_t, int* err, cudaStream_t st);
int ahb_ssd_state_bwd_tc(const void* Cm, const void* dy, const void* dec_t, const float* cl, int B, int L, int H,
                         const float* ds_final, void* dse_t, float* ds0, int* err, cudaStream_t st);
// chunk-parallel backward: one CTA per (chunk, batch, head group); dB_part / dC_part are (G, B, L, N)
// fp32 scratch with G = ahb_ssd_head_groups(H), summed into dB / dC; dA (H,) is accumulated (zero it)
int ahb_ssd_head_groups(int H);
// diagnostics: per-phase cycle counters of the scan kernels (uint64[64] per file or null; phase_prof.cuh)
int ahb_ssd_phase_prof(void* counters);
int ahb_gdn_phase_prof(void* counters);
int ahb_ssd_bwd_chunk_tc(const void* x, const void* dt, const float* A, const void* Bm, const void* Cm, const void* dy,
                         int B, int L, int H, const void* sin_t, const void* dse_t, const void* yd_t, void* dx, void* ddt,
                         float* dB, float* dC, float* dA, float* dB_part, float* dC_part, int* err, cudaStream_t st);

// moe_gemm.cu: tcgen05 grouped GEMM.  Returns 0 on success, <0 on a setup error.
#define AHB_GEMM_DENSE 0        // C[M,N] = A[M,K] B[N,K]^T (single group)
#define AHB_GEMM_FWD_SWIGLU 1   // h = silu(X W1_e) * (X W3_e); saves a1, a3
#define AHB_GEMM_FWD_GELU 2     // h = gelu(X W1_e); saves a1
#define AHB_GEMM_FWD_DOWN 3     // Y = H W2_e
#define AHB_GEMM_DH_SWIGLU 4    // dH = dY W2_e^T -> dA1, dA3
#define AHB_GEMM_DH_GELU 5      // dH = dY W2_e^T -> dA1
#define AHB_GEMM_DX 6           // dX = dA1 W1_e^T (+ dA3 W3_e^T)
#define AHB_GEMM_WGRAD 7        // dW_e += A_e^T B_e   (fp32 accumulate)
#define AHB_GEMM_WGRAD_DUAL 8   // dW1_e += X_e^T dA1_e, dW3_e += X_e^T dA3_e
// or-ed into the kind: run the CTA-pair kernel (cta_group::2, 256 x 256 tiles); M-grouped
// group offsets must then be multiples of 256 rows, K-grouped Mout a multiple of 256
#define AHB_GEMM_PAIR 0x100
// or-ed into a weight-gradient kind: the accumulators are bf16 (fp32 sums rounded once per add)
#define AHB_GEMM_ACC_BF16 0x200
int ahb_moe_gemm(int kind, const void* a0, const void* a1, int64_t a_rows, int64_t a_cols, const void* b0,
                 const void* b1, int64_t b_rows_total, int64_t b_cols, int b_rows_per_group, const int* grp_off,
                 int E, int N, int Mout, int K, int kb_split, void* out0, void* out1, void* out2, const void* aux0,
                 const void* aux1, float clip, int* err, int num_sms, cudaStream_t st,
                 const float* alpha = nullptr, int m_limit = 0);

// moe.cu: routing positions, gather / combine (+ backward)
// segments padded to multiples of `pad` rows (128, or 256 for the CTA-pair GEMMs)
void ahb_moe_route(const int* eidx, int T, int k, int E, int* counts, int* off, int* pos, int* row_src, int64_t R_cap,
                   cudaStream_t st, int pad = 128);
void ahb_moe_gather(const void* x, const int* row_src, int64_t R, int d, void* xs, cudaStream_t st);
void ahb_moe_zero_pad(void* m, const int* row_src, int64_t R, int d, cudaStream_t st);
void ahb_moe_combine(const void* ys, const int* pos, const float* gate, const void* shared, int T, int k, int d,
                     void* out, cudaStream_t st);
void ahb_moe_combine_bwd(const void* dout, const void* ys, const int* pos, const float* gate, int T, int k, int d,
                         void* dys, float* dgate, cudaStream_t st);
void ahb_moe_scatter_add(const void* dxs, const int* pos, int T, int k, int d, void* dx, cudaStream_t st);

// optim.cu: fused optimizer over the owned shard
#define AHB_LABEL_MUON 0
#define AHB_LABEL_LION 1
#define AHB_LABEL_ADAMW_DECAY 2
#define AHB_LABEL_ADAMW_NODECAY 3
#define AHB_LABEL_FROZEN 4
#define AHB_SEG_COMPUTE_FP32 1
#define AHB_SEG_ROUTER_TEMP 2
#define AHB_SEG_EXPERT_BIAS 4
#define AHB_SEG_REQUIRES_GRAD 8
struct AhbSegInfo {
  int64_t off;    // state-space offset relative to the owned shard
  int64_t coff;   // compute-space offset (16-bit units)
  int64_t len;
  int32_t label, group, flags, bias_row;
  float gscale;
  int32_t pad;
};
struct AhbOptimArgs {
  float lr[5];
  float wd[5];
  float bc1, bc2;
};
int ahb_optim_chunk();
// grad: fp32, or bf16 with grad_bf16 (a store with 16-bit gradient accumulators)
void ahb_optim_prepare(const AhbSegInfo* segs, const int* cstart, int S, int nblocks, void* grad, bool grad_bf16,
                       const float* master, float inv, double* red, int* flags, const float* const* gpeers,
                       int npeers, int64_t lo, cudaStream_t st);
void ahb_optim_apply(const AhbSegInfo* segs, const int* cstart, int S, int nblocks, float* master, float* m, float* v,
                     const void* grad, bool grad_bf16, const float* coef, void* compute, const float* frac, int fracE,
                     AhbOptimArgs args, void* const* cpeers, int npeers, cudaStream_t st);
// Muon Newton-Schulz update X <- nan_to_num(1.5 X - 0.5 Y), Xb <- bf16(X) (Y null: Xb only); n % 4 == 0
void ahb_ns_update(float* X, const void* Y, void* Xb, int64_t n, int num_sms, cudaStream_t st);

// fused_norm.cu: residual add + clip + RMSNorm, RMSNorm x SiLU gate, GDN gates, per-head L2 norm, Mamba2 dt
// (bf16 activations, fp32 scales / statistics; rows of D channels need D % 256 == 0)
int ahb_row_supported(int D);
int ahb_row_bwd_blocks(int64_t M);
void ahb_add_rmsnorm_fwd(const void* x, const void* delta, const float* scale, void* xo, void* y, float* rstd,
                         int64_t M, int D, float clip, float eps, cudaStream_t st,
                         float* stats = nullptr);
void ahb_add_rmsnorm_bwd(const void* dy, const void* gres, const void* xo, const float* scale, const float* rstd,
                         void* dx, void* ddelta, float* dscale_part, int64_t M, int D, float clip, cudaStream_t st);
void ahb_norm_gate_fwd(const void* x, const void* z, int64_t zs, const float* scale, void* y, float* rstd, int64_t M,
                       int D, float eps, float zclip, float oclip, cudaStream_t st);
void ahb_norm_gate_bwd(const void* dy, const void* x, const void* z, int64_t zs, const float* scale, const float* rstd,
                       void* dx, void* dz, float* dscale_part, int64_t M, int D, float zclip, float oclip,
                       cudaStream_t st);
// tensor-parallel (head-split) RMSNorm, gated when z is non-null: the row sums ss (forward) and dot
// (backward) are all-reduced over the group between the two passes of each direction
void ahb_tp_norm_sumsq(const void* x, float* ss, int64_t M, int D, cudaStream_t st);
void ahb_tp_norm_fwd(const void* x, const void* z, int64_t zs, const float* scale, const float* ss, void* y,
                     float* rstd, int64_t M, int D, float inv_dfull, float eps, float zclip, float oclip,
                     cudaStream_t st);
void ahb_tp_norm_bwd_dot(const void* dy, const void* x, const void* z, int64_t zs, const float* scale,
                         const float* rstd, void* dz, float* dot, float* dscale_part, int64_t M, int D, float zclip,
                         float oclip, cudaStream_t st);
void ahb_tp_norm_bwd_dx(const void* dy, const void* x, const void* z, int64_t zs, const float* scale,
                        const float* rstd, const float* dot, void* dx, int64_t M, int D, float inv_dfull, float zclip,
                        float oclip, cudaStream_t st);
void ahb_gdn_gates_fwd(const void* bp, const void* wp, const void* fp, const float* decay_a, void* bg, void* wg,
                       float* g, int64_t n, int d, int Dh, cudaStream_t st);
void ahb_gdn_gates_bwd(const void* dbg, const void* dwg, const float* dg, const void* bg, const void* wg,
                       const void* fp, const float* decay_a, void* dbp, void* dwp, void* dfp, float* da_acc,
                       int64_t n, int d, int Dh, cudaStream_t st);
void ahb_l2norm_heads_fwd(const void* x, void* y, float* rn, int64_t nheads, cudaStream_t st);
void ahb_l2norm_heads_bwd(const void* dy, const void* x, const float* rn, void* dx, int64_t nheads, cudaStream_t st);
void ahb_dt_act_fwd(const void* u, void* dt, int64_t n, cudaStream_t st);
void ahb_dt_act_bwd(const void* ddt, const void* u, void* du, int64_t n, cudaStream_t st);

// router.cu: fused cosine router (fp32-exact logits on tensor cores, clip, noise, biased top-k, gate
// softmax, aux/z statistics).  EP = ahb_router_padded_experts(E).
int ahb_router_supported(int d, int E, int k);
int ahb_router_padded_experts(int E);
// knT3: (3, EP, d) bf16 = hi/mid/lo terms of kn^T (zero padded);
// scal (5 floats, zero except scal[4] = +large): sum lse^2, max |pre-clip logit|, sum |x|, max |x|, min |x|
void ahb_router_fwd(const void* x, const void* knT3, const float* temp, const float* bias, const float* noise,
                    int64_t T, int d, int E, int k, float* logits, float* cosv, float* rn, int64_t* top_idx,
                    float* gate, float* probs_sum, float* scal, float* counts, cudaStream_t st);
// kn2: (2, d, EP) bf16 = hi/mid terms of kn; dcos: (T, EP) fp32 scratch; dtemp and dkn (d, E) accumulate
void ahb_router_bwd(const void* x, const void* kn2, const float* temp, const float* logits, const float* cosv,
                    const float* rn, const int64_t* top_idx, const float* gate, const float* dgate, const float* dps,
                    const float* dlse_sq, int64_t T, int d, int E, int k, float* dcos, float* dtemp, void* dx,
                    float* dkn, cudaStream_t st);

// ep.cu: expert-parallel token exchange over peer memory
void ahb_ep_publish(const int* counts, int E, int* const* peers_dev, int W, int rank, cudaStream_t st);
void ahb_ep_dispatch(const void* src, int src_by_token, int T, int k, int d, const int* eidx, const int* pos_local,
                     const int* off_local, const int* dst_base, int El, void* const* recv_peers,
                     void* const* meta_peers, int rank, int* dst_pos, cudaStream_t st);
void ahb_ep_return(const void* rows, const void* meta, int64_t R, int d, void* const* ret_peers, cudaStream_t st);
void ahb_ep_zero_pad(void* rows, void* meta, const int* off, const int* seg, int El, int d, cudaStream_t st);

// attention.cu: causal flash attention (q, k, v, o (BH, L, D) bf16, D in {64, 96, 128}); lse (BH, L) fp32.
// Backward: delta = rowsum(dO o O) (BH, L) fp32; dq (BH, L, D) fp32 accumulated (zero it first).
int ahb_attn_supported(int D);
int ahb_attn_fwd(const void* q, const void* k, const void* v, int BH, int L, int D, float scale, void* o, float* lse,
                 cudaStream_t st);
int ahb_attn_bwd(const void* q, const void* k, const void* v, const void* dout, const float* lse, const float* delta,
                 int BH, int L, int D, float scale, float* dq, void* dk, void* dv, cudaStream_t st);

// source_mix.cu: BlockDAR source softmax (out = sum_i softmax_i(scale <q, k_i>) s_i), pointer tables of n <= 32
int ahb_source_mix_max();
void ahb_source_mix_fwd(const void* q, const void* const* ks, const void* const* ss, int n, int64_t T, int dl, int d,
                        float scale, void* out, float* wts, cudaStream_t st);
void ahb_source_mix_bwd(const void* g, const void* q, const void* const* ks, const void* const* ss, const float* wts,
                        int n, int64_t T, int dl, int d, float scale, void* dq, void* const* dks, void* const* dss,
                        cudaStream_t st);

// comm.cu: NVLink peer-memory collectives (CUDA IPC buffers, bounded barriers)
int ahb_ipc_alloc(int64_t nbytes, void** ptr);
int ahb_ipc_free(void* ptr);
int ahb_ipc_handle(void* ptr, void* handle64);
int ahb_ipc_open(const void* handle64, void** ptr);
int ahb_ipc_close(void* ptr);
void ahb_symm_barrier(uint32_t* const* pads_dev, int rank, int world, uint32_t epoch, int* err, double timeout_s,
                      cudaStream_t st);
void ahb_reduce_scatter_f32(const float* const* peers_dev, int world, int64_t lo, int64_t n, float* out,
                            cudaStream_t st);
// acc (N,) += column sums of dy (M, N) with row stride ld (elements, a multiple of 8)
void ahb_bias_grad_acc(const void* dy, int64_t M, int N, int64_t ld, float* acc, cudaStream_t st);
// tensor parallelism over peer memory
int ahb_gemm_rs_peer(const void* a, int64_t a_rows, int64_t K, const void* b, int64_t N, const int* grp_off, int W,
                     void* const* out_tab, int m_rot, int* err, int num_sms, cudaStream_t st);
void ahb_sum_slots_bf16(const void* slots, int nslots, int64_t stride, int64_t n, void* out, cudaStream_t st);
int ahb_memcpy_async(void* dst, const void* src, int64_t nbytes, cudaStream_t st);
void ahb_copy_out(const void* src, void* const* peers_dev, int world, int64_t off_bytes, int64_t nbytes,
                  cudaStream_t st);

// ce.cu: label-smoothed cross entropy over bf16 logits rows, gradient written in place
// Dense projections on the grouped GEMM (moe_gemm.cu): mode 0 y = x W (+ bias) (+ beta_src), mode 1
// y = dy W^T (+ beta_src), mode 2 acc fp32 += x^T dy; grp_off = {0, M padded to the tile height}
int ahb_dense_gemm(int mode, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int K, int N,
                   const void* bias, const void* beta_src, void* out, const int* grp_off, int* err, int num_sms,
                   cudaStream_t st, bool pair);
// LM-head GEMM with a cross-entropy epilogue (moe_gemm.cu; see there), and the row combine of its
// forward partials: lse per row, sum of the label-smoothed losses and of the valid rows (ce.cu)
int ahb_ce_gemm(bool bwd, const void* h, int64_t rows, int d, const void* W, int V, const int* grp_off,
                const int64_t* labels, const float* lse, float ls, void* out, int* err, int num_sms, cudaStream_t st,
                bool pair);
void ahb_ce_combine(const void* partials, int ntiles, const int64_t* labels, int64_t T, int V, float ls, float* lse,
                    float* loss_sum, float* count, cudaStream_t st);
