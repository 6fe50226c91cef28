/*
 * dsca_b200 — C ABI of the B200 (sm_100a) MoE-block forward for DSCA-MoE.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream, launches its kernels
 * on that stream and returns an int status (DSCA_OK = 0).  Apart from the expert-parallel
 * symmetric region (dsca_ep_region_alloc, set-up time), nothing here allocates device
 * memory: buffers and scratch space come from the caller, with the shapes documented beside
 * each argument struct.  Kernels that detect a problem (a wait past its
 * time limit, an out-of-range index, more rows than the workspace holds) write a code into the
 * caller's device error word instead of trapping; dsca_check_error reads it back.
 *
 * References are to the acbling/DSCA-MoE source tree.
 */
#ifndef DSCA_B200_H_
#define DSCA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DSCA_API __attribute__((visibility("default")))
#else
#define DSCA_API
#endif

typedef struct CUstream_st* dsca_stream_t;

/* status codes */
enum {
  DSCA_OK = 0,
  DSCA_ERR_BAD_ARG = 1,       /* a null pointer, a bad size or an unsupported combination */
  DSCA_ERR_CAPACITY = 2,      /* more rows / experts / tokens than the kernel or buffer allows */
  DSCA_ERR_WAIT_TIMEOUT = 3,  /* a device-side wait passed its time limit (kernel returned) */
  DSCA_ERR_CUDA = 4,          /* a CUDA runtime or driver call failed */
  DSCA_ERR_DEVICE_INDEX = 5,  /* a kernel's bounds check rejected an index */
  DSCA_ERR_UNSUPPORTED = 6    /* not available on this device (needs sm_100) */
};

/* element types */
enum { DSCA_F32 = 0, DSCA_BF16 = 1, DSCA_F8E4M3 = 2 };

/* routing modes */
enum {
  DSCA_ROUTE_SWITCH_TOP1 = 0, /* softmax in the router dtype, argmax (first index on ties) */
  DSCA_ROUTE_SOFTMAX_TOPK = 1 /* softmax in fp32, top-k by (prob desc, expert id asc) */
};

/* expert activation */
enum {
  DSCA_ACT_RELU = 0,   /* Switch DenseActDense: wo(ReLU(wi x)) */
  DSCA_ACT_SWIGLU = 1  /* Qwen2MoeMLP: down(SiLU(gate x) * up x) */
};

/* Tokens routed by one router CTA; per-block histograms are [ceil(T / DSCA_ROUTER_TOKENS), E]. */
#define DSCA_ROUTER_TOKENS 32
/* Largest expert count the router handles in one warp (2 experts per lane). */
#define DSCA_MAX_EXPERTS 64
#define DSCA_MAX_TOPK 8
#define DSCA_MAX_GPUS 8

DSCA_API const char* dsca_version(void);
DSCA_API const char* dsca_status_string(int status);

/* Number of SMs of the current device and whether it is an sm_100 part (1) or not (0). */
DSCA_API int dsca_device_info(int* num_sms, int* is_sm100);

/*
 * Router: logits, softmax, top-k, per-block histogram and in-block stable ranks, fused.
 * Replaces Router.standard_forward (src/harmonymoe/router.py:52-63) with the argmax at
 * src/qosmoe/moe_layer.py:286-287, and the gate / softmax / topk of ShardedQwenMoE.forward
 * (qwen_ep_adapter/qwen_ep.py:48-53), plus the shared-expert gate sigmoid(x . g)
 * (qwen_ep_adapter/qwen_ep.py:94).
 * Arithmetic order is fixed (bit-identical to the C oracle): with the tensor-core fields below
 * (bf16 only), logit = the exact fixed-point dot product of the bf16 rows (21 bits below each
 * row's largest exponent, accumulated in integers on int8 tcgen05 MMAs), converted once to fp32
 * and rounded to bf16; otherwise the fp32 fma chains of the kernel's chunked order, rounded to
 * the dtype.  Softmax uses a deterministic exp.
 */
typedef struct {
  const void* x;              /* [T, d], dtype */
  const void* w_router;       /* [E, d], dtype (the reference router runs in its weight dtype) */
  const void* w_shared_gate;  /* [d] dtype, or NULL (no shared expert) */
  int T, d, E, top_k;
  int dtype;                  /* DSCA_F32 or DSCA_BF16, for x and the router weight */
  int mode;                   /* DSCA_ROUTE_* */
  int norm_topk;              /* divide the k weights by their sum (Qwen norm_topk_prob) */
  int weight_round_bf16;      /* round routing weights to bf16 (activation dtype bf16) */
  void* logits;               /* [T, E] dtype */
  int32_t* topk_ids;          /* [T, top_k] */
  float* topk_w;              /* [T, top_k] */
  int64_t* expert_index;      /* [T] top-1 id as int64, or NULL */
  float* shared_gate;         /* [T] sigmoid(round_dtype(x . g)), or NULL */
  int32_t* block_hist;        /* [ceil(T/32), E] tokens per expert in each 32-token block */
  int32_t* local_rank;        /* [T, top_k] rank of (t, j) among its block's tokens of that expert */
  /* optional fused scan (the dsca_dispatch_scan outputs, computed by the last CTA to finish):
     set all four, done_counter pointing at a zeroed uint32 that the kernel leaves at zero */
  int32_t* counts;            /* [E] */
  int32_t* offsets;           /* [E + 1] */
  int32_t* block_base;        /* [ceil(T/32), E] */
  uint32_t* done_counter;
  /* optional tensor-core logits (bf16): w_slices and w_exp select them; d16 = d rounded up to 16.
     d <= 2048 runs one fused kernel (clusters of four CTAs per 128 tokens) and needs no scratch;
     a larger d needs the three scratch buffers as well (NULL otherwise) */
  const void* w_slices;       /* [3][64][d16] int8 from dsca_router_pack_i8 */
  const int32_t* w_exp;       /* [64] from dsca_router_pack_i8 */
  void* x_slices;             /* [3][T][d16] int8 scratch (d > 2048) */
  int32_t* x_exp;             /* [T] scratch (d > 2048) */
  float* logits_f32;          /* [T][64] scratch (d > 2048) */
  int32_t* err;               /* device error word for the tensor-core pass's bounded waits, or NULL */
  /* optional: first_counts[e] += how many of the tokens chose e first (integer atomics; the
     QoS planner's n(e), dsca_qos_args.first_counts, which zeroes it again), or NULL */
  int32_t* first_counts;
} dsca_router_args;
DSCA_API int dsca_router_topk(const dsca_router_args* a, dsca_stream_t stream);

/*
 * Router rows for the tensor-core logits: `rows` [R][d] bf16 (R <= 64: the E router rows, then
 * the shared-expert gate row) -> three int8 slice planes [3][64][d16] and the rows' exponents
 * [64]; rows R..63 are zero.  Run once per router weight.
 */
DSCA_API int dsca_router_pack_i8(const void* rows, int R, int d, void* w_slices, int32_t* w_exp,
                                 dsca_stream_t stream);

/*
 * Dispatch scan: per-expert counts, expert-major row offsets and each block's base rank inside
 * every expert.  Replaces the bincount / sort / nonzero lists of
 * src/qosmoe/moe_layer.py:206-215,300-304 and qwen_ep_adapter/qwen_ep.py:62,69,80.
 */
typedef struct {
  const int32_t* block_hist;  /* [nblocks, E] */
  int nblocks, E;
  int32_t* counts;            /* [E] */
  int32_t* offsets;           /* [E + 1] exclusive prefix of counts */
  int32_t* block_base;        /* [nblocks, E] tokens of expert e in blocks before b */
} dsca_scan_args;
DSCA_API int dsca_dispatch_scan(const dsca_scan_args* a, dsca_stream_t stream);

/*
 * Permute: copy each routed (token, slot) row of x into the send / expert-major buffer.
 * Row of (t, j) with expert e and per-expert rank q = block_base[b][e] + local_rank[t][j]:
 * the destination dst is the first with q < cum_split[e][dst] (cumulative plan S[rank, e, :]),
 * and the row is dest_base[e][dst] + q - cum_split[e][dst-1].  With one GPU, pass
 * cum_split = NULL: the row is offsets[e] + q.  This is the a8 order of
 * Scheduler.distribute_tokens (src/harmonymoe/scheduler.py:101-124): destination ascending,
 * expert ascending, token ascending inside the expert, earliest tokens to the lowest dst.
 */
typedef struct {
  const void* x;              /* [T, d] */
  int T, d, E, top_k, dtype;
  const int32_t* topk_ids;    /* [T, k] */
  const int32_t* local_rank;  /* [T, k] */
  const int32_t* block_base;  /* [nblocks, E] */
  const int32_t* offsets;     /* [E + 1] (one-GPU layout) */
  int G;                      /* GPUs in the plan (1 = local layout) */
  const int32_t* cum_split;   /* [E, G] inclusive prefix over dst of S[rank, e, :], or NULL */
  const int32_t* dest_base;   /* [E, G] first send row of (e, dst), or NULL */
  int capacity;               /* rows of `out` */
  void* out;                  /* [capacity, d] */
  int32_t* token_row;         /* [T, k] row written for (t, j) */
  int32_t* err;               /* device error word */
  int out_f16;                /* bf16 input: write the rows as f16 (fp8-weight FFN operand) */
  void* x_f16;                /* [T, d] f16 copy of x (shared-expert operand), or NULL */
  int out_e4m3;               /* bf16 input: write each row as two e4m3 terms (dsca_split_rows;
                                 2 * Kd bytes a row, Kd = d rounded up to 128) with its 1 / s in
                                 out_scale[row] (operand of the f8_split FFN) */
  float* out_scale;           /* [capacity] */
  void* x_q;                  /* [T, 2 * Kd] two-term copy of x (shared-expert operand), or NULL */
  float* x_scale;             /* [T] */
} dsca_permute_args;
DSCA_API int dsca_permute(const dsca_permute_args* a, dsca_stream_t stream);

/*
 * Grouped expert FFN.  Replaces the per-expert loop tokens[idx] = expert(tokens[idx])
 * (src/qosmoe/async_cpu.py:137-173, src/qosmoe/moe_layer.py:226-253,
 * qwen_ep_adapter/qwen_ep.py:85-89) and the shared expert (qwen_ep.py:94).
 * bf16: tcgen05 grouped GEMM (TMEM accumulators, TMA-fed 128B-swizzled tiles, persistent
 * tile scheduler over (group, M tile, N tile) read from device-side offsets).
 * f32: CUDA-core grouped GEMM (fp32 parity mode).
 * Weights are packed once (dsca_moe_b200 python: pack_*):
 *   SwiGLU w1: [E, N1p, d] with N1p = 2 * ceil(I/128) * 128; each 256-row block holds 128 gate
 *              rows then the 128 matching up rows (zero rows past I).
 *   ReLU   w1: [E, N1p, d] with N1p = ceil(F/256) * 256 (zero rows past F).
 *   w2:        [E, dp, Ip] with dp = ceil(d/256) * 256, Ip = N1p/2 (SwiGLU) or N1p (ReLU),
 *              zero past d rows / I columns.
 * h holds the activated intermediate [rows, Ip]; y the expert outputs [rows, d].
 */
typedef struct {
  int dtype;                  /* DSCA_BF16 (tcgen05) or DSCA_F32 (CUDA cores) */
  int act;                    /* DSCA_ACT_* */
  int d;                      /* model width: GEMM1 K, GEMM2 N */
  int n1p;                    /* packed GEMM1 N per expert */
  int ip;                     /* packed intermediate width (GEMM2 K) */
  int dp;                     /* packed GEMM2 N per expert */
  int num_groups;             /* row groups in `a` */
  const int32_t* group_offsets; /* device [num_groups + 1] row offsets into a / h / y */
  const int32_t* group_weight;  /* device [num_groups] expert index into w1 / w2, NULL = identity */
  int num_experts_w;          /* experts in w1 / w2 */
  int capacity;               /* rows of a / h / y */
  const void* a;              /* [capacity, d] */
  const void* w1;             /* [num_experts_w, n1p, d] */
  const void* w2;             /* [num_experts_w, dp, ip] */
  void* h;                    /* [capacity, ip] */
  void* y;                    /* [capacity, d] */
  /* optional shared expert on all T tokens (Qwen): same packing with E = 1 */
  int shared_rows;            /* 0 = none */
  int shared_n1p, shared_ip;
  const void* xs;             /* [shared_rows, d] */
  const void* ws1;            /* [shared_n1p, d] */
  const void* ws2;            /* [dp, shared_ip] */
  void* hs;                   /* [shared_rows, shared_ip] */
  void* ys;                   /* [shared_rows, d] */
  int32_t* err;               /* device error word */
  int num_ctas;               /* persistent CTAs (0 = one per SM) */
  int phases;                 /* 0 or 3 = both GEMMs; 1 = GEMM1 only; 2 = GEMM2 only */
  void* ep_ctx;               /* expert-parallel context (dsca_ep_init), or NULL: when set, GEMM2
                                 stores each routed output row straight into the return buffer of
                                 the rank that sent it and sets that rank's return flag */
  int segments;               /* 0 or 3 = routed and shared; 1 = routed only; 2 = shared only */
  /* dtype = DSCA_F8E4M3: w1 / w2 / ws1 / ws2 hold e4m3 bytes and these per-output-channel fp32
     scales (one per packed weight row: [E * n1p], [E * dp], [shared_n1p], [dp]); a, xs, h and hs
     are f16 (e4m3 converts exactly to f16 for the kind::f16 MMA), y and ys bf16. */
  const float* w1_scale;
  const float* w2_scale;
  const float* ws1_scale;
  const float* ws2_scale;
  int tile_rows;              /* bf16 path tile form: 128 = one CTA per 128-token x 256-channel
                                 tile; 256 = a CTA pair (tcgen05 cta_group::2) per 256-channel x
                                 <=256-token tile, tokens rounded up to 16 only; 512 = CTA pairs,
                                 and in a SwiGLU GEMM1 every whole 256-token block of a group is
                                 one non-swapped tile (256 tokens x the gate and up rows of 128
                                 channels), the rest as in 256; 0 = default (pair for GEMM2 and
                                 ReLU GEMM1, single CTA for SwiGLU GEMM1).
                                 dtype DSCA_F8E4M3: 256 = the weights converted into tensor memory
                                 (e4m3 -> f16 by converter warps, the MMA's A operand read from
                                 TMEM, tokens as the MMA N); anything else = the weights converted
                                 into shared memory */
  int pdl_after_permute;      /* 1: the call directly follows dsca_permute on the same stream (one
                                 GPU): GEMM1 is launched as the permute's programmatic dependent
                                 (with a shared expert its tiles go first and overlap the permute;
                                 the routed tiles wait on the device for the permute), and GEMM2 as
                                 GEMM1's (it waits for GEMM1's outputs before its first load) */
  const int32_t* group_order; /* device [num_groups]: execution order of the routed groups
                                 (position -> group; a permutation), or NULL = index order.  The
                                 QoS planner's order (dsca_ep_group_order); bf16 only, other dtypes
                                 run index order.  Only the order of the tiles changes, never a
                                 result */
  int cache_hints;            /* bf16 and f8_split.  Bit 0: 0 = default L2 policy for every load;
                                 1 = the routed experts' weights (streamed from DRAM, mostly read
                                 once) loaded evict-first, the shared expert's weights and the
                                 token rows evict-last.  Bits 8-15: L2 prefetch distance in K
                                 blocks for the routed tiles' operands (0 = off) */
  int tile_order;             /* bit 0, routed and shared expert in one launch (bf16): 0 = one
                                 segment's tiles after the other's (the default); 1 = their tiles
                                 interleaved in proportion to their counts (after one round of
                                 shared tiles when GEMM1 overlaps the permute), HBM-bound routed
                                 tiles beside tensor-bound shared tiles.  Bits 1 / 2: the shared
                                 expert's / the routed groups' tiles weight-block major (every
                                 token block of one weight block, then the next weight block)
                                 instead of token-block major.  No bit changes a result. */
  /* dtype DSCA_F8E4M3 with f8_split = 1: the e4m3 weights go to the tensor cores as they are
     (tcgen05 kind::f8f6f4, CTA-pair tiles with the tokens as the MMA N), multiplied by tokens held
     as two e4m3 terms per value (dsca_split_rows): a [capacity, 2 * Kd] and xs [shared_rows,
     2 * Kd] bytes (Kd = d rounded up to 128) with 1 / s per row in a_scale and xs_scale.  GEMM1
     writes h and hs in bf16; the call splits them into hq [capacity, 2 * ip] and hsq
     [shared_rows, 2 * shared_ip] with h_scale and hs_scale, which GEMM2 reads; y and ys bf16.
     ep_ctx must be NULL. */
  int f8_split;
  const float* a_scale;
  const float* xs_scale;
  void* hq;
  void* hsq;
  float* h_scale;
  float* hs_scale;
  /* optional dynamic tile schedule: 8 zeroed uint32 (GEMM1 uses [0, 2), GEMM2 [2, 4), the
     shared-expert handoff [4, 6)), left zeroed by every call.  Each CTA (pair) then takes its next
     tile from an atomic ticket when it is ready for one, so tiles of different lengths spread by
     their actual durations; NULL = the static schedule.  Calls that overlap on the GPU must not
     share them. */
  uint32_t* tile_counters;
  /* 1: with tile_counters, both phases in this call, pdl_after_permute, bf16 SwiGLU in the
     default tile form and a shared expert, GEMM1 raises a flag once its shared-expert tiles are
     stored and GEMM2's shared-expert tiles start on it instead of after all of GEMM1 (GEMM2's
     CTAs take the SMs GEMM1's CTAs leave); otherwise ignored.  0 = off. */
  int shared_handoff;
} dsca_ffn_args;
DSCA_API int dsca_grouped_ffn(const dsca_ffn_args* a, dsca_stream_t stream);

/*
 * Two-term e4m3 rows (the token operand of the f8_split FFN; no counterpart in the reference,
 * whose experts run in the weights' dtype).  Each bf16 row x of src [rows, ld] is scaled by a
 * power of two s (its largest magnitude to [128, 256)) and written as hi = RN_e4m3(s x) and
 * lo = RN_e4m3(s x - hi): dst row = [hi: Kp bytes | lo: Kp bytes], Kp = K rounded up to 128,
 * zero past K; inv_scale[row] = 1 / s.  hi + lo = s x exactly for |s x| >= 1/4.  One warp a row;
 * rows_dev (device int, or NULL) bounds the rows processed.
 */
typedef struct {
  const void* src;            /* bf16 [rows, ld] */
  int ld, rows, K;            /* K % 8 == 0, K <= ld, ld % 8 == 0 */
  const int32_t* rows_dev;    /* device row count (min with rows), or NULL */
  void* dst;                  /* [rows, 2 * Kp] bytes */
  float* inv_scale;           /* [rows] */
} dsca_split_args;
DSCA_API int dsca_split_rows(const dsca_split_args* a, dsca_stream_t stream);

/*
 * Grouped expert FFN for callers that cannot allocate device memory (no counterpart in the
 * reference).  Same arguments and results as dsca_grouped_ffn for bf16 and f32, except that `h`
 * and `hs` must be NULL: the GEMM1 intermediate lives in a fixed array inside this library, so a
 * caller that runs where cudaMalloc is unavailable or forbidden (inside a graph replay or a
 * callback, or under a foreign, already-full allocator) only passes its inputs and outputs.
 * dtype DSCA_F8E4M3, and ep_ctx with DSCA_F32, return DSCA_ERR_UNSUPPORTED.
 * Limit: capacity * ip + shared_rows * shared_ip elements (plus 256-byte alignment of the first
 * part) must fit in DSCA_STATIC_SCRATCH_BYTES, else DSCA_ERR_CAPACITY; `phases` must be 0 or 3.
 * Every GPU that loads the library holds that many bytes until exit.  The first call on a device
 * (and the first after a device reset) looks the array up with that device current; make it
 * before any stream capture.  All calls share the array: calls that overlap on the GPU race;
 * calls ordered on one stream are safe.
 */
#define DSCA_STATIC_SCRATCH_BYTES (16u << 20)
DSCA_API int dsca_grouped_ffn_static_scratch(const dsca_ffn_args* a, dsca_stream_t stream);

/*
 * Combine: out[t] = sum_j w[t,j] * y[token_row[t,j]] (+ shared_gate[t] * ys[t]), summed in
 * fp32 in slot order and rounded once.  Replaces router_probs * h (src/qosmoe/moe_layer.py:
 * 255-258) and the index_add_ + shared-expert add of qwen_ep_adapter/qwen_ep.py:92-94 with a
 * deterministic gather (no atomics).
 */
typedef struct {
  int T, d, top_k, dtype;
  const void* y;              /* [rows, d] expert outputs */
  const int32_t* token_row;   /* [T, k] */
  const float* topk_w;        /* [T, k] */
  const void* ys;             /* [T, d] shared expert output, or NULL */
  const float* shared_gate;   /* [T] or NULL */
  int rows;                   /* rows of y (bounds check) */
  void* out;                  /* [T, d] */
  int32_t* err;
  int pdl;                    /* 1: the call directly follows dsca_grouped_ffn on the same stream;
                                 the combine is launched as its programmatic dependent (its blocks
                                 start early and wait on the device for GEMM2's outputs) */
} dsca_combine_args;
DSCA_API int dsca_combine(const dsca_combine_args* a, dsca_stream_t stream);

/*
 * QoS planner scores.  Replaces QoSPlanner.compute_token_scores and aggregate_expert_priority
 * (src/qosmoe/planner.py:63-170).  They change no result: the expert-cache path orders its
 * experts and chooses what to load by them (build_exec_plan, :172-237, on the host).  Per token:
 *   gain    = |x - x_prev| (|x| when x_prev is NULL)
 *   attn    = population variance of the token's logits row (0 when attention_mode = 1)
 *   penalty = target_batch / (n(e0) + epsilon), e0 = the token's first choice, n(e) = how many
 *             of the T tokens chose e first
 *   score   = seq_priority (1 + gain (1 + attn) / (alpha d + beta remaining + delta penalty)),
 *             -1e9 where valid == 0
 * and per expert the sum of the scores of its (token, slot) assignments.  NULL per-token
 * vectors read as seq_priority 1, remaining 0, valid 1.
 */
typedef struct {
  const void* x;              /* [T, d] block input */
  const void* x_prev;         /* [T, d] previous layer's hidden states, or NULL */
  const void* logits;         /* [T, E] router logits */
  int dtype;                  /* of x, x_prev and logits: DSCA_BF16 or DSCA_F32 */
  const int32_t* topk_ids;    /* [T, top_k], first choice first */
  const float* seq_priority;  /* [T] or NULL */
  const float* remaining;     /* [T] or NULL */
  const float* valid;         /* [T] or NULL */
  int T, d, E, top_k;
  int attention_mode;         /* 0 = router_var, 1 = none */
  float alpha, beta, delta, target_batch, epsilon;
  float* token_score;         /* [T] */
  float* expert_priority;     /* [E] */
  int32_t* err;
  /* optional one-kernel form (set partial and done_counter): every 32-token CTA scores its tokens
     and sums its own assignments per expert into partial; the last CTA to finish adds the
     partials in CTA order into expert_priority (the same result whatever the schedule).
     first_counts: n(e) accumulated by dsca_router_topk in the same forward, read here and left
     zeroed for the next forward; NULL = counted here from topk_ids */
  int32_t* first_counts;      /* [E] or NULL */
  float* partial;             /* [ceil(T / 32), E] scratch, or NULL */
  uint32_t* done_counter;     /* zeroed uint32 that the kernel leaves at zero, or NULL */
} dsca_qos_args;
DSCA_API int dsca_qos_priority(const dsca_qos_args* a, dsca_stream_t stream);

/*
 * Harmony plan on the host (integer, deterministic, identical on every rank).
 * Restates Scheduler.schedule_harmony (src/harmonymoe/scheduler.py:324-372) over an arbitrary
 * expert -> GPU placement (the exflow [layer][gpu] -> experts format,
 * src/harmonymoe/scheduler.py:51-64,230-237, converted to expert_to_gpu).  eq_tokens < 0 gives
 * schedule_fixed (:268-279).  One guard is added: an outer pass that moves nothing ends the
 * loop (the reference would spin there).  meta: [G, E] counts; S: [G, E, G] out.
 */
DSCA_API int dsca_plan_harmony(const int32_t* meta, int G, int E, const int32_t* expert_to_gpu,
                      int eq_tokens, int32_t* S);

/*
 * Receive layout for rank `rank` from plan S [G, E, G] (host arrays): the groups are the
 * experts with tokens for this rank in ascending id; inside a group, chunks of src ascending
 * (the stable form of Scheduler.generate_expert_mask, src/harmonymoe/scheduler.py:185-213).
 * Outputs: num_groups, group_expert[E], group_offsets[E + 1], recv_off[G, E] (row of chunk
 * (src, e) in the expert-major receive buffer, -1 if empty), and for the sender side
 * send_base[E, G] (first send row of (e, dst) on `rank`), cum_split[E, G], send_splits[G],
 * recv_splits[G].
 */
DSCA_API int dsca_plan_layout(const int32_t* S, int G, int E, int rank, int* num_groups,
                     int32_t* group_expert, int32_t* group_offsets, int32_t* recv_off,
                     int32_t* send_base, int32_t* cum_split, int32_t* send_splits,
                     int32_t* recv_splits);

/*
 * Fused expert-parallel exchange over NVLink (one process per GPU).  Each rank owns a symmetric
 * region: flags [3][DSCA_MAX_GPUS] u32, meta [2][DSCA_MAX_GPUS][DSCA_MAX_EXPERTS] (i32 counts,
 * then fp32 priorities), a receive
 * buffer [recv_capacity, d] and a return buffer [ret_capacity, d]; every rank maps every peer's
 * region (dsca_ipc_export / dsca_ipc_import) and passes the G pointers of each part.
 * Per forward, on one stream, with no host synchronisation:
 *   dsca_ep_plan      counts -> every peer, bounded wait for all counts, harmony plan and send /
 *                     receive tables on the device (replaces the metadata all_to_all and
 *                     Scheduler.schedule_harmony, src/qosmoe/moe_layer.py:367-385);
 *   dsca_ep_dispatch  rows stored straight into the destination ranks' expert-major receive
 *                     buffers, then the dispatch flag (replaces distribute_tokens + the dispatch
 *                     all_to_all_single, moe_layer.py:393-408);
 *   dsca_ep_wait      bounded wait for a flag kind from every peer (kind 0 counts, 1 dispatch,
 *                     2 return);
 *   dsca_grouped_ffn  with ep_ctx set (the return all_to_all fused into GEMM2's epilogue,
 *                     moe_layer.py:435-440);
 *   dsca_combine      over the local return buffer.
 * Every wait gives up after limit_ns and records DSCA_ERR_WAIT_TIMEOUT in the error word.
 */
typedef struct {
  int G, E, me, d, elem_bytes;
  int recv_capacity, ret_capacity;
  int eq_tokens;                  /* harmony threshold; < 0 = fixed placement */
  unsigned int start_epoch;       /* the same on every rank (0 on a freshly zeroed region) */
  const int32_t* expert_to_gpu;   /* host [E] */
  void* flags[DSCA_MAX_GPUS];     /* per rank p: p's flag array (this process's mapping) */
  void* meta[DSCA_MAX_GPUS];
  void* recv[DSCA_MAX_GPUS];
  void* ret[DSCA_MAX_GPUS];
} dsca_ep_setup;
DSCA_API size_t dsca_ep_ctx_bytes(void);
DSCA_API int dsca_ep_init(void* ctx_dev, const dsca_ep_setup* s, dsca_stream_t stream);
/* Device pointer of the plan's receive-side group offsets [E + 1] inside ctx_dev. */
DSCA_API int32_t* dsca_ep_group_offsets(void* ctx_dev);
/* Device pointer of the QoS execution order [E] inside ctx_dev (position -> expert), written by
 * dsca_ep_plan or dsca_ep_priority: experts by their priority summed over the ranks, descending,
 * lowest id on ties (the priority all-reduce and build_exec_plan order of
 * src/qosmoe/moe_layer.py:379-380,422-427); the identity after a dsca_ep_plan without
 * priorities.  Pass it as dsca_ffn_args.group_order. */
DSCA_API int32_t* dsca_ep_group_order(void* ctx_dev);
/* Copy the last plan S [DSCA_MAX_GPUS][DSCA_MAX_EXPERTS][DSCA_MAX_GPUS] and the rows this rank
 * received to the host (synchronises `stream`; for statistics, not the hot path). */
DSCA_API int dsca_ep_read_plan(void* ctx_dev, int32_t* S_host, int32_t* recv_total_host, dsca_stream_t stream);
/* priority: this rank's expert priorities [E] (dsca_qos_priority), or NULL (identity order) */
DSCA_API int dsca_ep_plan(void* ctx_dev, const int32_t* counts, const float* priority, uint64_t limit_ns,
                          int32_t* err, dsca_stream_t stream);
/* dsca_ep_plan split in two for a forward whose dispatch should not wait for the QoS scores
 * (the harmony plan and the layouts need only the counts; the priorities only order the routed
 * tiles): dsca_ep_plan_counts is dsca_ep_plan without the execution order (left as it is), and
 * dsca_ep_priority exchanges this rank's priorities [E] with every peer (bounded wait), sums them
 * in rank order and writes the execution order (dsca_ep_group_order).  Once each per forward on
 * every rank, in any order or concurrently on different streams; the GEMM that reads the order
 * must come after dsca_ep_priority.  Same reference lines as dsca_ep_plan. */
DSCA_API int dsca_ep_plan_counts(void* ctx_dev, const int32_t* counts, uint64_t limit_ns, int32_t* err,
                                 dsca_stream_t stream);
DSCA_API int dsca_ep_priority(void* ctx_dev, const float* priority, uint64_t limit_ns, int32_t* err,
                              dsca_stream_t stream);
typedef struct {
  const void* x;
  int T, d, top_k, dtype;
  const int32_t* topk_ids;
  const int32_t* local_rank;
  const int32_t* block_base;
  void* ctx;                  /* device context */
  int32_t* token_row;         /* [T, k] out: row of (t, j) in this rank's return buffer */
  int32_t* err;
  int out_f16;                /* bf16 input: store the rows as f16 (the fp8-weight FFN operand) */
  void* x_f16;                /* [T, d] f16 copy of x written here (shared-expert operand), or NULL */
} dsca_ep_dispatch_args;
DSCA_API int dsca_ep_dispatch(const dsca_ep_dispatch_args* a, dsca_stream_t stream);
DSCA_API int dsca_ep_wait(void* ctx_dev, int kind, uint64_t limit_ns, int32_t* err, dsca_stream_t stream);
/* Return path as its own kernel (when GEMM2 stored routed rows locally into y [rows, d]): row r
 * of this rank's receive layout is stored into its source rank's return buffer, one warp per row
 * (contiguous 512-byte NVLink stores), then the return flag is set at every peer.  max_rows
 * bounds the launch (the receive capacity); the row count itself is read on the device. */
DSCA_API int dsca_ep_return(void* ctx_dev, const void* y, int d, int dtype, int max_rows, int32_t* err,
                            dsca_stream_t stream);
/* The device harmony plan on its own (test hook): meta, e2g, S are device arrays. */
DSCA_API int dsca_ep_plan_eval(const int32_t* meta, int G, int E, const int32_t* expert_to_gpu,
                               int eq_tokens, int32_t* S, dsca_stream_t stream);
/* The one set-up-time allocation of this library: a rank's symmetric region, its own cudaMalloc
 * block (zeroed) so that CUDA IPC maps exactly that block into the peers.  Freed by
 * dsca_ep_region_free after every peer closed its mapping. */
DSCA_API int dsca_ep_region_alloc(size_t bytes, void** ptr);
DSCA_API int dsca_ep_region_free(void* ptr);
/* CUDA IPC of a device allocation (any pointer inside it): 64-byte handle + offset. */
DSCA_API int dsca_ipc_export(const void* ptr, void* handle64, size_t* offset);
DSCA_API int dsca_ipc_import(const void* handle64, size_t offset, void** ptr);
DSCA_API int dsca_ipc_close(void* ptr, size_t offset);

/* Read (and clear) the device error word; returns the matching DSCA_ERR_* or DSCA_OK.
 * Synchronises `stream`. */
DSCA_API int dsca_check_error(int32_t* err_dev, dsca_stream_t stream);

/* Device-side exp used by routing, evaluated on n inputs (test hook for the oracle pin). */
DSCA_API int dsca_exp_neg_eval(const float* x, float* y, int n, dsca_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DSCA_B200_H_ */
