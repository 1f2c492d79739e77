/*
 * kolibri_b200.h — C ABI of libkolibri_b200.so, the sm_100a implementation of the
 * non-GEMM MoE decode hot path of Kolibri-style decoders (router, expert maps,
 * activation expansion, Q/K RMSNorm + RoPE, sandwich / post-MoE residual norms).
 *
 * Conventions shared by every entry point
 *  - All pointers are device pointers unless stated otherwise; buffers are dense,
 *    row-major and must not alias unless an entry point says so.
 *  - Every call is asynchronous on `stream` (0 = legacy default stream), performs no
 *    host synchronisation and no device allocation; every scratch buffer is passed in.
 *  - Return value: KB_OK (0) on success; a negative KB_ERR_* for an invalid argument,
 *    shape, dtype, alignment or workspace size (nothing was launched); a positive
 *    value is a cudaError_t reported by the launch.
 *  - Floating point: no fast-math.  expf/sqrtf/division are the IEEE-accurate CUDA
 *    forms, so results track the PyTorch eager CPU path within the tolerances the
 *    tests state.
 */
#ifndef KOLIBRI_B200_H
#define KOLIBRI_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KB_API __attribute__((visibility("default")))
#else
#define KB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t (driver_types.h declares `struct CUstream_st *`). */
typedef struct CUstream_st *kb_stream_t;

enum {
    KB_OK = 0,
    KB_ERR_INVALID_ARG = -1,  /* null pointer, negative size, bad flag           */
    KB_ERR_UNSUPPORTED = -2,  /* shape / dtype / K / E outside the kernel's range */
    KB_ERR_ALIGNMENT = -3,    /* pointer or row stride not aligned as required    */
    KB_ERR_WORKSPACE = -4,    /* workspace missing or smaller than *_workspace_bytes */
    KB_ERR_TOO_LARGE = -5,    /* T*K or row count overflows the int32 index space */
    KB_ERR_SCRATCH_LIMIT = -6 /* kb_expert_maps_noalloc: request exceeds its static scratch */
};

/* Element types of activation tensors. */
enum { KB_BF16 = 0, KB_F16 = 1, KB_F32 = 2 };

/* Expert-map algorithm selection (`mode` argument). */
enum {
    KB_MAPS_AUTO = 0,        /* single CTA at small T, persistent multi-CTA kernel above   */
    KB_MAPS_SINGLE_CTA = 1,  /* one CTA, everything in shared memory (T*K <= 12288)         */
    KB_MAPS_MULTI_CTA = 2,   /* persistent cooperative kernel (two-kernel path if it cannot hold T) */
    KB_MAPS_TWO_KERNEL = 3,  /* tile histograms + per-super-tile scatter, two launches      */
    /* Forced multi-CTA routing paths of kb_router_maps (kb_expert_maps treats them as
     * KB_MAPS_MULTI_CTA): the fallbacks AUTO takes when the tile kernel does not apply. */
    KB_MAPS_HYBRID_ROUTER = 4,  /* lane-per-token hybrid router kernel (E in {128..512})    */
    KB_MAPS_WARP_ROUTER = 5     /* warp-per-token router kernel (any E <= 512, K <= 32)       */
};

KB_API const char *kb_status_str(int status);
KB_API int kb_version(void);

/* ---------------------------------------------------------------------------------
 * Failure detection.  Every wait inside the multi-CTA kernels (grid barriers, bulk-copy
 * barriers, the decode chain's logit all-gather) is bounded.  A wait that gives up sets its
 * workspace's error word and the call returns early with invalid outputs; every later call on
 * that workspace writes offsets[0..E] = -1 and nothing else until the workspace is zero-filled
 * again (kb_expert_maps_noalloc: flags = KB_NOALLOC_REZERO).
 * kb_workspace_status reads the error word (it waits for `stream` first):
 *   kind   KB_WS_MAPS (kb_expert_maps / kb_router_maps workspace), KB_WS_CHAIN
 *          (kb_decode_chain workspace), KB_WS_NOALLOC (the static scratch of
 *          kb_expert_maps_noalloc on the current device; workspace is ignored), KB_WS_EP
 *          (a rank's expert-parallel exchange buffer, section (e) below), KB_WS_RGEMM
 *          (kb_router_gemm workspace)
 *   status KB_WS_CLEAN (0), KB_WS_TIMEOUT (1: a bounded wait gave up),
 *          KB_WS_MISALIGNED (2: kb_decode_chain found a layer weight pointer that is not
 *          16-byte aligned), KB_WS_CAPACITY (3: an expert-parallel exchange received more
 *          rows than its buffer holds, or a rank's counts were invalid)
 * kb_set_wait_limit sets the number of polls after which every later launch's waits give up
 * (0 restores the defaults, about a second of polling); it returns the previous setting.  A
 * short limit makes waits give up early on purpose, so that the error path can be exercised.
 * No counterpart in the reference (its kernels report launch errors only,
 * kernels/cuda/customKolibriBuildExpertMapsKernel.cu:78-88). */
enum { KB_WS_MAPS = 0, KB_WS_CHAIN = 1, KB_WS_NOALLOC = 2, KB_WS_EP = 3, KB_WS_RGEMM = 4 };
enum { KB_WS_CLEAN = 0, KB_WS_TIMEOUT = 1, KB_WS_MISALIGNED = 2, KB_WS_CAPACITY = 3 };
KB_API int kb_workspace_status(const void *workspace, int kind, int *status, kb_stream_t stream);
KB_API long long kb_set_wait_limit(long long polls);
/* Programmatic dependent launch on (1, default) or off (0) for every later launch
 * made by this library in this process.  Returns the previous value. */
KB_API int kb_set_pdl(int enable);

/* ---------------------------------------------------------------------------------
 * (a1) Router: scores = logits + bias; ids = top-K of scores (descending, the lower
 * expert index wins ties, NaN ranks above +inf as in torch.sort); weights =
 * sigmoid(logits[ids]) of the UN-biased logit; if renorm, weights /= (sum + 1e-20).
 *   logits fp32 [T, E] (row stride E), bias fp32 [E] or NULL (= zero bias),
 *   ids int32 [T, K], weights [T, K] in w_dtype (KB_F32, KB_BF16 or KB_F16).
 *   1 <= K <= 32, K <= E <= 512.
 * Replaces: kolibri_gate_forward (kernels/cuda/customKolibriRoutingKernels.cu:238-266,
 * bound by kernels/cuda/router_bindings.cpp:60-104) and _fused_kolibri_router_kernel
 * (kernels/triton/fused_kolibri_router.py:38-95, launched at :98-146); renorm=1 is the
 * prologue router invokeKolibriRouter (fusions/03_moe_prologue/fused/custom_moe_prologue.cu:104-119).
 */
KB_API int kb_router(const float *logits, const float *bias, int32_t *ids, void *weights,
              int w_dtype, int64_t T, int E, int K, int renorm, kb_stream_t stream);

/* ---------------------------------------------------------------------------------
 * (a2) Expert maps from top-K ids [T, K] (int32, row-major, selection s = t*K + k).
 *   counts   int32 [E]     (may be NULL)   number of selections of each expert
 *   offsets  int64 [E+1]   exclusive scan of counts; offsets[E] = number of valid ids
 *   p2u      int32 [T*K]   permuted row -> unpermuted row, unpermuted row = k*T + t
 *                          (slot-major), rows sorted by (expert, token, slot);
 *                          entries past offsets[E] are set to -1
 *   u2p      int32 [T*K]   (may be NULL) inverse: u2p[k*T + t] = permuted row; -1 for
 *                          an id outside [0, E)
 * Ids outside [0, E) are skipped, as the reference kernels skip them.
 * The workspace must be zero-filled before its first use; every call leaves it
 * zero-filled again (its arrival counters reset themselves).
 * Replaces: invokeKolibriBuildExpertMaps (kernels/cuda/customKolibriBuildExpertMapsKernel.cu:37-89,
 * bound at kernels/cuda/build_expert_maps_bindings.cpp:10-40), invokeKolibriMultiBlockBuildExpertMaps
 * (kernels/cuda/multi_block_expert_maps/customKolibriMultiBlockBuildExpertMapsKernels.cu:36-213)
 * and invokeDynamicBuildExpertMaps (fusions/03_moe_prologue/fused/custom_moe_prologue.cu:409-444).
 */
KB_API size_t kb_expert_maps_workspace_bytes(int64_t T, int E, int K);
KB_API int kb_expert_maps(const int32_t *ids, int32_t *counts, int64_t *offsets, int32_t *p2u,
                   int32_t *u2p, void *workspace, size_t workspace_bytes, int64_t T,
                   int E, int K, int mode, kb_stream_t stream);

/* (a1)+(a2) in one pass over the logits: router outputs (as kb_router, weights fp32)
 * and the expert maps (as kb_expert_maps) of the ids it selects.
 * Replaces the router + map stages of invokeFusedMoePrologue
 * (fusions/03_moe_prologue/fused/custom_moe_prologue.cu:524-547). */
KB_API size_t kb_router_maps_workspace_bytes(int64_t T, int E, int K);
KB_API int kb_router_maps(const float *logits, const float *bias, int32_t *ids, float *weights,
                   int32_t *counts, int64_t *offsets, int32_t *p2u, int32_t *u2p,
                   void *workspace, size_t workspace_bytes, int64_t T, int E, int K,
                   int renorm, int mode, kb_stream_t stream);

/* The path kb_expert_maps (route = 0) or kb_router_maps (route = 1) takes for this shape:
 * *path = KB_MAPS_SINGLE_CTA, KB_MAPS_MULTI_CTA (persistent kernel; with route = 1 the tile
 * kernel), KB_MAPS_HYBRID_ROUTER / KB_MAPS_WARP_ROUTER (route = 1: those router kernels) or
 * KB_MAPS_TWO_KERNEL,
 * *launches = kernel launches per call, *grid = CTAs of the (first) launch.  Any output
 * pointer may be NULL.  Library introspection; no counterpart in the reference. */
KB_API int kb_maps_describe(int64_t T, int E, int K, int route, int mode, int *path,
                            int *launches, int *grid);

/* (f3) Router projection on the tensor cores with the routing fused into its epilogue:
 *   logits[t, e] = bf16(sum_h x[t, h] * w_gate[e, h]) widened to fp32 (fp32 accumulation,
 *   one rounding: the `(x @ W_g).float()` of a bf16 GEMM), then ids / weights from those
 *   logits exactly as kb_router (bias, top-K, sigmoid of the rounded logit, renorm option).
 *   x       bf16 [T, H] row-major, 16-byte aligned
 *   w_gate  bf16 [E, H] row-major (the nn.Linear layout: logits = x @ w_gate^T), 16-byte aligned
 *   bias    fp32 [E] or NULL;  logits fp32 [T, E] or NULL (not stored)
 *   ids     int32 [T, K] or NULL (no routing: logits only);  weights fp32 [T, K]
 *   H % 64 == 0, E % 64 == 0, E <= 512, 1 <= K <= 8, T <= 524288 (else KB_ERR_TOO_LARGE).
 * The workspace (kb_router_gemm_workspace_bytes(T, H, E, K), 256-byte aligned) must be
 * zero-filled before its first use; every call leaves its counters at zero.  A bounded wait
 * that gives up sets its error word (kb_workspace_status kind KB_WS_RGEMM); the workspace must
 * then be zero-filled again.  The hidden dimension is split over several CTAs when T is small
 * (their fp32 partials are summed in split order, so results do not depend on timing).
 * Replaces the gate GEMM + router of the reference's layer: gate_gemm and R2_moe_prologue of
 * benchmarks/11_profile_2block_e2e.py:236-246 (torch.matmul on cuBLAS, then
 * fused_moe_prologue / the routing kernels of (a1)). */
KB_API size_t kb_router_gemm_workspace_bytes(int64_t T, int H, int E, int K);
KB_API int kb_router_gemm(const void *x, const void *w_gate, const float *bias, float *logits,
                          int32_t *ids, float *weights, void *workspace, size_t workspace_bytes,
                          int64_t T, int H, int E, int K, int renorm, kb_stream_t stream);
/* The tile shape kb_router_gemm takes for this shape: *bn experts per CTA tile, *ks hidden
 * splits, *grid CTAs.  Any output pointer may be NULL.  Library introspection; no counterpart
 * in the reference. */
KB_API int kb_router_gemm_describe(int64_t T, int H, int E, int K, int *bn, int *ks, int *grid);

/* kb_expert_maps (mode KB_MAPS_AUTO, same outputs and rules) for callers that may not
 * allocate device memory: its workspace is a static 8 MiB device array inside this
 * library (one per device), so neither the caller nor the library allocates anything.
 * No counterpart in the reference (which allocates its scratch with torch per call).
 *   Who needs it: hosts whose contract forbids allocation in the launch path, e.g. an
 *   inference engine that hands all free HBM to its KV cache after a profiling pass (a
 *   later cudaMalloc fails or fragments), or a plugin enqueue() that may only use the
 *   workspace its host sized up front.
 *   Limits: T <= 524288 tokens and a workspace bound (kb_expert_maps_workspace_bytes)
 *   <= 8 MiB, which holds for every E <= 512, K <= 32 at that T; a larger request
 *   returns KB_ERR_SCRATCH_LIMIT and launches nothing.
 *   First call on each device: resolves the scratch address with cudaGetSymbolAddress
 *   (the CUDA runtime loads this library's device code then if it has not yet) and
 *   zero-fills the scratch on `stream`.  Make it before any stream capture; a call with
 *   T = 0 does only this set-up and zeroes offsets (and counts).
 *   Zero state: the scratch must hold zeros when a call starts; every completed call
 *   leaves it so.  If a bounded wait inside the kernel gave up (offsets all -1), pass
 *   flags = KB_NOALLOC_REZERO on the next call to zero-fill it again first.
 *   Device: the scratch used is the CURRENT device's; `stream` must belong to that device
 *   (a stream of another device returns KB_ERR_INVALID_ARG).
 *   Concurrency: all calls on one device share the scratch.  Calls must be ordered
 *   (one stream, or streams joined by events); two calls in flight at once on the same
 *   device race on the scratch and give wrong maps.
 */
enum { KB_NOALLOC_REZERO = 1 };
KB_API int kb_expert_maps_noalloc(const int32_t *ids, int32_t *counts, int64_t *offsets,
                                  int32_t *p2u, int32_t *u2p, int64_t T, int E, int K,
                                  int flags, kb_stream_t stream);

/* ---------------------------------------------------------------------------------
 * Activation expansion: out[r] = x[p2u[r] % T] for r in [0, rows); a row whose p2u
 * is negative or >= rows_total_unpermuted is left untouched.  row_bytes is the row
 * size in bytes (any element type).  16-byte aligned rows take the vector path.
 * Replaces: invokeKolibriActivationExpansion (fusions/03_moe_prologue/fused/custom_moe_prologue.cu:481-501)
 * and invokeKolibriActivationExpansionFromMap (kernels/cuda/customKolibriBuildExpertMapsKernel.cu:197-222).
 */
KB_API int kb_expand_rows(const void *x, void *out, const int32_t *p2u, int64_t T, int64_t rows,
                   int64_t row_bytes, kb_stream_t stream);
/* The expansion of T*K rows together with the permuted routing weights, in one pass:
 * out[r] = x[p2u[r] % T] and scales[r] = weights[(p2u[r] % T)*K + p2u[r] / T] (fp32 [T*K];
 * 0 for a row past offsets[E], whose p2u is -1).  row_bytes a multiple of 16, x and out
 * 16-byte aligned.  Replaces the permuted_scales gather of the router-dispatch entry point
 * (kernels/cuda/router_dispatch_bindings.cpp:62-126, kernels/cuda/kolibri_router_dispatch.py:49-64). */
KB_API int kb_expand_rows_scaled(const void *x, void *out, const int32_t *p2u,
                                 const float *weights, float *scales, int64_t T, int K,
                                 int64_t row_bytes, kb_stream_t stream);

/* MoE finalize (combine), the consumer of the maps and weights:
 *   out[t, :] = dtype( sum_{k < K} float(expert_out[u2p[k*T + t], :]) * weights[t, k] )
 * fp32 products, summed in slot order k = 0..K-1, one rounding to dtype; a slot whose u2p is
 * negative or >= T*K contributes nothing.  expert_out [T*K, H] in permuted (expert) order,
 * u2p int32 [K*T] (kb_expert_maps), weights fp32 [T, K], out [T, H]; dtype KB_BF16, KB_F16
 * or KB_F32; rows 16-byte aligned.  1 <= K <= 32.
 * Replaces the eager finalize of the reference harness
 * (benchmarks/11_profile_2block_e2e.py:259-262). */
KB_API int kb_moe_finalize(const void *expert_out, const int32_t *u2p, const float *weights,
                           void *out, int64_t T, int K, int64_t H, int dtype, kb_stream_t stream);

/* ---------------------------------------------------------------------------------
 * (a4) Per-head Q/K RMSNorm fused with NeoX RoPE, bf16 in and out:
 *   y = x * (1/sqrt(mean(x^2) + eps)) * gamma     (fp32, per head of D elements)
 *   a_j = float(pos[t]) * inv_freq[j], j < D/2
 *   out = [y1*cos(a) - y2*sin(a), y2*cos(a) + y1*sin(a)]  -> bf16 (one rounding)
 * pos == NULL selects the RNoPE layers' identity rotation (pure per-head RMSNorm).
 * q: [T, Hq, D] with token stride q_tok_stride elements (>= Hq*D), same for k.
 * q_out/k_out may equal q_in/k_in (in place).  D is 64, 128 or 256.
 * inv_freq fp32 [D/2] on the device = 1/theta^(2j/D), computed by the caller.
 * Replaces: TensorRT-LLM fusedQKNormRopeKernel as driven by Kolibri1Attention.apply_rope
 * (benchmarks/02_benchmark_attention_norm.py:105-112); formula of
 * scratch/diag_rope_fusion.py:31-38; RNoPE = per-head F.rms_norm of
 * benchmarks/11_profile_2block_e2e.py:195-196.
 */
KB_API int kb_qk_norm_rope(const void *q_in, void *q_out, const void *k_in, void *k_out,
                    const void *gamma_q, const void *gamma_k, const int32_t *pos,
                    const float *inv_freq, int64_t T, int Hq, int Hkv, int D,
                    int64_t q_tok_stride, int64_t k_tok_stride, float eps,
                    kb_stream_t stream);

/* ---------------------------------------------------------------------------------
 * (a5)/(a6) Residual norm pair, rows of H elements of `dtype`:
 *   sum_out  = residual + RMSNorm(a) * g1        (rounded to dtype, then reused)
 *   norm_out = RMSNorm(sum_out) * g2
 * As the sandwich norm: a = attn_out, residual = residual_in -> (updated_residual, moe_in)
 *   Replaces invokeFusedSandwichNormReg (fusions/01_sandwich_norm/fused/custom_sandwich_norm.cu:120-158);
 *   oracle fusions/01_sandwich_norm/baseline/trtllm_baseline.py:78-95.
 * As the post-MoE + pre-attention norm: a = moe_out, residual = h -> (out, next)
 *   (benchmarks/11_profile_2block_e2e.py:229-231 applied after :269-270).
 * sum_out may alias residual; norm_out may alias a.
 */
KB_API int kb_residual_norm_pair(const void *a, const void *residual, const void *g1,
                          const void *g2, void *sum_out, void *norm_out, int64_t T,
                          int64_t H, float eps, int dtype, kb_stream_t stream);

/* Add + RMSNorm: sum = a + b (rounded to dtype); out = RMSNorm(sum) * g;
 * sum_out (may be NULL) receives sum.
 * Replaces invokeFusedAddPostMoeNorm (fusions/02_post_moe_norm/fused/custom_post_moe_norm.cu:194-228);
 * oracle fusions/02_post_moe_norm/baseline/trtllm_baseline.py:77-90.  With sum_out it is also
 * the decoder's input_layernorm (benchmarks/11_profile_2block_e2e.py:229-231). */
KB_API int kb_add_rms_norm(const void *a, const void *b, const void *g, void *out, void *sum_out,
                    int64_t T, int64_t H, float eps, int dtype, kb_stream_t stream);

/* ---------------------------------------------------------------------------------
 * (a7) The non-GEMM decode chain of n_layers layers in ONE launch, for decode batches
 * of 1 <= T <= 4 tokens (bf16 activations, head_dim 128, K <= 8, E <= 512, H <= 6144).
 * Per layer l, in the order of the reference harness's decoder_layer
 * (benchmarks/11_profile_2block_e2e.py:215-266; layer types of config.json:29-80):
 *   q_out, k_out  = Q/K RMSNorm + RoPE of q, k (as kb_qk_norm_rope; rnope: no rotation)
 *   h, moe_in     = sandwich of attn_out and the residual stream (as kb_residual_norm_pair)
 *   logits        = float(bf16(moe_in @ w_gate_t^T))   (router GEMV, fp32 accumulation)
 *   ids, weights, counts, offsets, p2u, u2p = router + expert maps of logits (as
 *                   kb_router_maps with renorm = 0)
 *   permuted      = expansion of moe_in by p2u (as kb_expand_rows)
 *   residual, next = post-MoE pair of moe_out and h (as kb_residual_norm_pair)
 * attn_out, moe_out, q and k are the outputs of the attention / expert GEMMs, which are
 * outside this library: the same buffers feed every layer.  The residual stream starts as
 * residual_in and ends in residual_out (which may alias it); no other output may overlap an
 * input (KB_ERR_INVALID_ARG).  h, moe_in, next, q_out, k_out, logits, ids, weights, maps and
 * permuted hold the last layer's values.  trace_logits (NULL or fp32 [n_layers, T, E])
 * receives every layer's logits.  `layers` is a DEVICE array of n_layers descriptors whose
 * weight pointers are 16-byte aligned (the bias 4-byte aligned).  pos == NULL makes every
 * layer RNoPE.
 * Launch: one cooperative launch of one CTA per SM.  Every CTA runs every stage on whole rows;
 * the CTAs meet once per layer, in the all-gather of the router GEMV's logits (each CTA owns
 * ceil(E / SMs) <= 4 experts).  Calls must not overlap other work that needs every SM.
 * Workspace (kb_decode_chain_workspace_bytes, 16-byte aligned): zero-fill it once before the
 * first call; later calls keep it consistent (a call epoch and the logit records live there),
 * so successive calls on one workspace must be ordered (one stream).
 * Failure contract: every wait inside the kernel is bounded.  If one gives up (or a layer's
 * weight pointer is misaligned), the call sets the workspace's error word, writes offsets[0..E]
 * = -1 and its other outputs are invalid; every later call on that workspace does nothing but
 * write offsets = -1 until the workspace is zero-filled again.  kb_workspace_status reads the
 * error word.
 * No single counterpart in the reference: it chains the entry points above.
 */
typedef struct {
    const void *g_post_attn;  /* bf16 [H] post-attention RMSNorm weight   */
    const void *g_pre_moe;    /* bf16 [H] pre-MoE RMSNorm weight           */
    const void *g_post_ffn;   /* bf16 [H] post-MoE RMSNorm weight          */
    const void *g_input_ln;   /* bf16 [H] next layer's input RMSNorm weight */
    const void *g_q;          /* bf16 [128] per-head q norm weight          */
    const void *g_k;          /* bf16 [128] per-head k norm weight          */
    const void *w_gate_t;     /* bf16 [E, H] router weight (nn.Linear layout) */
    const float *gate_bias;   /* fp32 [E] or NULL                           */
    int32_t rnope;            /* non-zero: full-attention layer, no RoPE    */
    int32_t reserved;
} kb_chain_layer_t;

KB_API size_t kb_decode_chain_workspace_bytes(void);
KB_API int kb_decode_chain(const kb_chain_layer_t *layers, int n_layers, const void *attn_out,
                           const void *moe_out, const void *q, const void *k,
                           const int32_t *pos, const float *inv_freq,
                           const void *residual_in, void *residual_out, void *h, void *moe_in,
                           void *next, void *q_out, void *k_out, float *logits, int32_t *ids,
                           float *weights, int32_t *counts, int64_t *offsets, int32_t *p2u,
                           int32_t *u2p, void *permuted, float *trace_logits, void *workspace,
                           size_t workspace_bytes, int64_t T, int H, int Hq, int Hkv, int D,
                           int E, int K, float eps, kb_stream_t stream);

/* ---------------------------------------------------------------------------------
 * (e) Expert-parallel exchange over peer memory: one process per GPU on one node; rank r of N
 * routes its own tokens and owns experts [r*E/N, (r+1)*E/N).  Every rank allocates one
 * exchange buffer (kb_ep_alloc, kb_ep_buffer_bytes), exports it (kb_ipc_export), and maps every
 * other rank's buffer (kb_ipc_import) into a kb_ep_group_t; the transfers are then plain stores
 * of this GPU's kernels into the peers' buffers over NVLink / NVSwitch, followed by release
 * increments of the receivers' arrival counters.  No host round trip and no NCCL call: the
 * splits and the destination rows are derived on the device from the all-gathered counts, so
 * every call below is asynchronous and can be captured in a CUDA graph.
 *
 * The calls are collective: every rank makes the same sequence of kb_ep_* calls on its own
 * stream (one rank's call waits, bounded, for the others).  Per MoE layer:
 *   kb_router_maps -> kb_ep_counts_allgather -> kb_ep_dispatch -> expert GEMMs on the rows
 *   of kb_ep_recv_rows (segments recv_offsets) -> kb_ep_combine.
 * Row order on the owner: by local expert, then by sending rank, then in the sender's
 * permuted (expert, token, slot) order -- the order an all-to-all of the expert-sorted rows
 * followed by a stable grouping by local expert produces.
 *
 * Failure contract: every wait is bounded (kb_set_wait_limit; by default about ten seconds
 * of polling, since a peer may start late).  A wait that gives up, or counts that exceed the
 * buffer's capacity, set the error word of this rank's buffer (kb_workspace_status with
 * KB_WS_EP and workspace = buf[rank]: KB_WS_TIMEOUT or KB_WS_CAPACITY); every later kb_ep_*
 * call on the group then returns at once (kb_ep_counts_allgather writes gathered = -1), and
 * the peers' waits for this rank give up in turn.  Recovery is a new group (fresh buffers).
 * The reference runs on one GPU and has no such path; the exchange follows the per-expert
 * counts of its maps (kernels/cuda/customKolibriBuildExpertMapsKernel.cu:96-156) and the
 * finalize of its harness (benchmarks/11_profile_2block_e2e.py:259-262). */
#define KB_MAX_RANKS 8
#define KB_IPC_HANDLE_BYTES 64
typedef struct {
    int world;                 /* number of ranks N, 1 <= N <= KB_MAX_RANKS                 */
    int rank;                  /* this process's rank                                        */
    int num_experts;           /* E (a multiple of N, <= 512)                                */
    int top_k;                 /* K (<= 32)                                                  */
    int64_t max_tokens;        /* largest token count of any rank's call                     */
    int64_t row_bytes;         /* bytes of one activation row (a multiple of 16)             */
    void *buf[KB_MAX_RANKS];   /* every rank's exchange buffer as mapped in this process
                                  (buf[rank] = this rank's own, from kb_ep_alloc)            */
} kb_ep_group_t;

/* Size of one rank's exchange buffer (identical on every rank for identical arguments):
 * control words, the tagged count rows, N*max_tokens*K received rows, max_tokens*K returned
 * rows.  kb_ep_alloc allocates it with cudaMalloc on the current device and zero-fills it
 * (set-up call: synchronous, the only allocation in this library); kb_ep_free releases it. */
KB_API size_t kb_ep_buffer_bytes(int world, int E, int K, int64_t max_tokens, int64_t row_bytes);
KB_API int kb_ep_alloc(size_t bytes, void **buf);
KB_API int kb_ep_free(void *buf);
/* CUDA IPC export of a kb_ep_alloc buffer into KB_IPC_HANDLE_BYTES host bytes, and the
 * mapping of a peer's exported buffer into this process (peer access enabled on first use). */
KB_API int kb_ipc_export(const void *buf, void *handle);
KB_API int kb_ipc_import(const void *handle, void **buf);
KB_API int kb_ipc_close(void *buf);

/* gathered[q*E + e] = counts[e] of rank q (int32 [N, E]).  One CTA: it stores this rank's
 * counts, tagged with the call's epoch, into every rank's buffer and waits for every rank's
 * row (two slots by epoch parity).  Replaces the ncclAllGather of counts. */
KB_API int kb_ep_counts_allgather(const kb_ep_group_t *g, const int32_t *counts,
                                  int32_t *gathered, kb_stream_t stream);
/* kb_router_maps on this rank's T tokens (E and K of the group) followed by
 * kb_ep_counts_allgather of its counts, with the all-gather fused into the router + maps kernel
 * on its single-CTA path (decode T) and its tile path (large T): one launch, the counts leave
 * for every rank as soon as the expert totals are known and the kernel's last CTA collects
 * every rank's row; the other paths take two launches.  Outputs as kb_router_maps, plus
 * gathered int32 [N, E]. */
KB_API int kb_router_maps_allgather(const kb_ep_group_t *g, const float *logits,
                                    const float *bias, int32_t *ids, float *weights,
                                    int32_t *counts, int64_t *offsets, int32_t *p2u,
                                    int32_t *u2p, void *workspace, size_t workspace_bytes,
                                    int64_t T, int renorm, int mode, int32_t *gathered,
                                    kb_stream_t stream);
/* Device-side barrier of the group: returns (on the stream) once every rank has entered its
 * own call, so the work queued after it starts on every GPU at about the same time (used to
 * align the ranks before a timed region). */
KB_API int kb_ep_barrier(const kb_ep_group_t *g, kb_stream_t stream);
/* Sends this rank's routed rows to their owners: permuted row r (expert e, source token
 * p2u[r] % T of x [T, row_bytes]) goes straight to its final grouped row on rank e/(E/N) --
 * the expansion, the pack and the all-to-all in one pass.  recv_offsets int64 [E/N + 1]:
 * segments of this rank's local experts in its received rows (kb_ep_recv_rows).  Returns
 * when this rank's rows are sent and every rank's rows for this rank have arrived.
 * gathered is this call's kb_ep_counts_allgather output; p2u the maps of the same routing. */
KB_API int kb_ep_dispatch(const kb_ep_group_t *g, const void *x, int64_t T, const int32_t *p2u,
                          const int32_t *gathered, int64_t *recv_offsets, kb_stream_t stream);
/* Device address of this rank's received rows ([N*max_tokens*K, row_bytes] capacity; the
 * first recv_offsets[E/N] rows are valid after kb_ep_dispatch). */
KB_API int kb_ep_recv_rows(const kb_ep_group_t *g, void **rows);
/* Returns the expert outputs to their origins and finalizes there: expert_out holds this
 * rank's grouped rows (same order and count as its received rows; it may be the received
 * rows themselves); each goes back to the sender's permuted position, then
 *   out[t, :] = dtype( sum_k float(back[u2p[k*T + t], :]) * weights[t, k] )
 * exactly as kb_moe_finalize.  T, u2p and weights are this rank's, from the same routing as
 * the preceding kb_ep_dispatch; dtype KB_BF16, KB_F16 or KB_F32 (row_bytes = H * size). */
KB_API int kb_ep_combine(const kb_ep_group_t *g, const void *expert_out, const int32_t *gathered,
                         int64_t T, const int32_t *u2p, const float *weights, void *out,
                         int dtype, kb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KOLIBRI_B200_H */
