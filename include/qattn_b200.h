/*
 * qattn_b200.h — C ABI of the B200 (sm_100a) tree-verification kernels.
 *
 * Every entry point takes raw device pointers, element strides and sizes,
 * launches asynchronously on the given CUDA stream (a `cudaStream_t` passed
 * as `void*`; NULL = legacy default stream) and returns a status code:
 * QA_OK (0) or a negative QA_ERR_* value. Argument errors are detected on the
 * host before any launch; nothing throws across this boundary. No entry point
 * allocates device memory unless its comment says so; outputs are caller-owned.
 *
 * The Python layer (qattention_b200.ragged_attn) binds these with ctypes and
 * keeps the reference's operator API (src/ragged_attn.py of QAttention).
 */
#ifndef QATTN_B200_H
#define QATTN_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define QA_API __attribute__((visibility("default")))
#else
#define QA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define QA_OK 0
#define QA_ERR_INVALID (-1)     /* bad size, depth, branching factor, null pointer */
#define QA_ERR_UNSUPPORTED (-2) /* head_dim / dtype combination not compiled */
#define QA_ERR_ALIGN (-3)       /* pointer or stride breaks the 16-byte row rule */
#define QA_ERR_LAUNCH (-4)      /* CUDA launch error (cudaGetLastError) */
#define QA_ERR_DEVICE (-5)      /* no usable sm_100 device */

#define QA_DTYPE_F16 0
#define QA_DTYPE_BF16 1

/*
 * Ancestor-walk attention (tree part of tree verification).
 *
 * Replaces the Triton kernels behind
 *   ragged_attention            src/ragged_attn.py:1080-1166 (kernel :267-387)
 *   ragged_attention_with_lse   src/ragged_attn.py:499-572   (kernel :401-496)
 *   ragged_attention_with_parents src/ragged_attn.py:716-795 (kernel :593-713)
 * and the tree half of ragged_attention_hybrid (src/ragged_attn.py:1851-1888).
 *
 * For query token i (sequence-local) of sequence s, head h, the walk visits
 *   a_0 = i,  a_{t+1} = parent(a_t)   for t = 0 .. max_depth-1,
 * skipping a step whose node equals the previous step's node, where
 *   parent(a) = max(a-1, 0) / branching        (parents == NULL)
 *   parent(a) = parents[cu_q[s] + a]            (explicit; root self-loop)
 * and computes O = softmax_j(scale * q·K[a_j]) · V[a_j] in fp32.
 *
 * Layout: Q/O rows [T_q, Hq, D]; K/V rows [T_kv, Hkv, D] with the innermost
 * (D) stride 1. KV row of node a of sequence s is
 *   (cu_kv ? cu_kv[s] : cu_q[s]) + kv_offset + a.
 * GQA: query head h reads KV head h / (Hq / Hkv).
 *
 * Optional outputs/inputs:
 *   lse        fp32 [T_q, Hq] natural-log LSE of the result (NULL = skip)
 *   prefix_o / prefix_lse: a previously computed attention result over other
 *              keys (e.g. the shared prefix). When non-NULL it is merged in
 *              with the log-sum-exp rule of fused_lse_merge
 *              (src/ragged_attn.py:1576-1616); O and lse then describe the
 *              union of both key sets. prefix_o may alias o.
 */
/* Paged K/V (replaces ragged_attention_paged, src/ragged_attn.py:827-1047): when
 * page_table != NULL, K and V are caches [pages, page_size, kv_heads, D] and the KV row of
 * sequence b's node n (plus kv_offset) is slot (n % page_size) of physical page
 * page_table[b * page_table_stride + n / page_size]; k/v_stride_t are then the slot
 * strides and k/v_stride_page the page strides (elements). Every mode takes a page
 * table: complete trees (tensor-core tiles), chains (branching 1) and explicit parents
 * (the per-query walk).
 * Batched queries: q_stride_b = 0 reads query rows packed at cu_seqlens_q; a nonzero
 * q_stride_b places the query row of sequence b's node n at b*q_stride_b + n*q_stride_t
 * (a [B, N, H, D] view of any batch pitch, read in place; o and lse stay packed). */
typedef struct qa_ancestor_args {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;                  /* optional */
  const int32_t* cu_seqlens_q; /* [batch+1], device */
  const int32_t* cu_seqlens_kv;/* [batch+1], device, optional */
  const int32_t* parents;      /* [T_q], device, optional */
  const void* prefix_o;        /* optional, same dtype as o */
  const float* prefix_lse;     /* optional */
  int64_t q_stride_t, q_stride_h;
  int64_t k_stride_t, k_stride_h;
  int64_t v_stride_t, v_stride_h;
  int64_t o_stride_t, o_stride_h;
  int64_t lse_stride_t, lse_stride_h;
  int64_t prefix_o_stride_t, prefix_o_stride_h;
  int64_t prefix_lse_stride_t, prefix_lse_stride_h;
  int32_t batch;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;      /* 32, 64, 128 or 256 */
  int32_t kv_offset;     /* added to every KV row index (hybrid layout: L) */
  int32_t branching;     /* >= 1; ignored when parents != NULL */
  int32_t max_depth;     /* >= 0 */
  int32_t max_seqlen;    /* >= longest sequence in cu_seqlens_q */
  float scale;           /* softmax scale, the reference uses 1/sqrt(D) */
  int32_t dtype;         /* QA_DTYPE_F16 / QA_DTYPE_BF16 */
  const int32_t* page_table;    /* paged K/V: [batch, max_pages], device, optional */
  int64_t page_table_stride;    /* elements between sequences' rows of page_table */
  int64_t k_stride_page, v_stride_page;  /* paged K/V: elements between pages */
  int32_t page_size;            /* paged K/V: tokens per page */
  int64_t q_stride_b;           /* 0: packed query rows; else batch stride (see above) */
  void* workspace;              /* explicit parents: plan scratch (see below), optional */
  int64_t workspace_bytes;
  int32_t workspace_planned;    /* 1: workspace already holds the plans of these parents */
} qa_ancestor_args;

QA_API int qa_ancestor_attn(const qa_ancestor_args* args, void* stream);

/*
 * Explicit parents on tensor cores (ragged_attention_with_parents, the
 * reference's _ragged_attn_parents_kernel_lse, src/ragged_attn.py:593-795):
 * with parents != NULL and a device workspace of at least *bytes (16-byte
 * aligned) in args->workspace / workspace_bytes, qa_ancestor_attn plans every
 * (sequence, 64-query tile) from parents[] in a first kernel and runs the
 * tensor-core tiles on those plans; without it (or when *bytes is 0: head_dim
 * not 64/128/256, sequences over 16384 tokens, walks over 31 steps) it runs the
 * per-query walk. The plans depend on cu_seqlens_q, parents, max_depth,
 * max_seqlen and batch only: qa_ancestor_plan writes them alone, and a call with
 * workspace_planned = 1 reuses them (e.g. every layer of one verify step, which
 * share the draft tree) instead of planning again.
 */
QA_API int qa_ancestor_workspace_bytes(const qa_ancestor_args* args, int64_t* bytes);
QA_API int qa_ancestor_plan(const qa_ancestor_args* args, void* stream);

/*
 * Two-way log-sum-exp merge. Replaces fused_lse_merge
 * (src/ragged_attn.py:1619-1653, kernel :1576-1616):
 *   m = max(la, lb); wa = e^(la-m); wb = e^(lb-m)
 *   out = (wa*out_a + wb*out_b) / max(wa+wb, 1e-8)
 * Shapes [B, H, N(, D)] given by strides (elements) for b, h, n; D stride 1.
 * Unlike the reference it takes permuted views without a .contiguous() copy.
 */
QA_API int qa_lse_merge(const float* lse_a, const float* lse_b, const void* out_a,
                 const void* out_b, void* out, int32_t B, int32_t H, int32_t N,
                 int32_t head_dim, const int64_t* lse_a_strides /*[3]*/,
                 const int64_t* lse_b_strides /*[3]*/,
                 const int64_t* out_a_strides /*[3]*/,
                 const int64_t* out_b_strides /*[3]*/,
                 const int64_t* out_strides /*[3]*/, int32_t dtype, void* stream);

/*
 * Shared-prefix pass: attention of each sequence's N tree queries over its L
 * prefix keys (all prefix keys visible to every query), on tcgen05 tensor
 * cores. Replaces the dense part of tree verification: aten flash SDPA after
 * repeat_kv in scripts/w4a16_e2e.py:1236-1253 / :1446-1447, and the tl.dot
 * prefix loop of _ragged_attn_hybrid_kernel (src/ragged_attn.py:1761-1800).
 *
 * Tensors are [batch, tokens, heads, head_dim] with element strides for the
 * batch, token and head dimensions (head_dim stride 1; strides multiples of 8
 * elements; 16-byte aligned bases). GQA: query head h uses KV head
 * h / (num_q_heads / num_kv_heads); the group size must divide 128.
 * Writes O (same dtype) and the natural-log LSE (fp32, optional). The result
 * merges with the ancestor pass through qa_ancestor_args.prefix_o/prefix_lse.
 * head_dim 64 or 128; prefix_len >= 1.
 */
typedef struct qa_prefix_args {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse; /* optional */
  int64_t q_stride_b, q_stride_t, q_stride_h;
  int64_t k_stride_b, k_stride_t, k_stride_h;
  int64_t v_stride_b, v_stride_t, v_stride_h;
  int64_t o_stride_b, o_stride_t, o_stride_h;
  int64_t lse_stride_b, lse_stride_t, lse_stride_h;
  int32_t batch;
  int32_t num_queries; /* N: tree queries per sequence */
  int32_t prefix_len;  /* L: prefix keys per sequence */
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  float scale;
  int32_t dtype;
} qa_prefix_args;

QA_API int qa_prefix_attn(const qa_prefix_args* args, void* stream);

/*
 * W4A16 GEMM: Y[M, N] (fp16, row stride y_stride) = X[M, K] (fp16, row stride
 * x_stride) . dequant(W)[K, N], int4 weights with zero point 8, group 128
 * along K, fp16 scales. Replaces the GPTQModel Marlin W4A16 linears of the
 * verify step (scripts/w4a16_e2e.py:698-699; checkpoint format
 * scripts/quantize_llama31.py:41-59: bits=4, group_size=128, sym, no act-order).
 * Layout: qweight int32, tile-major [N/128][K/128][4][128][4]: each 128-column x
 * 128-k tile is one contiguous 8 KB block stored chunk-plane-major: index
 * [tn][tk][c][j][w] is output column 128 tn + j, word 4c + w of its row, which
 * holds k = 8 (4c + w) .. + 7 with k%8 = 2i in nibble i and k%8 = 2i+1 in nibble i+4;
 * scales fp16 [K/128, N]. K % 128 == 0, N % 128 == 0, 16-byte aligned pointers.
 * splits: K split across CTAs (0 = automatic, see qa_w4a16_plan). With more
 * than one split, `workspace` (fp32, splits*M*N elements, caller-allocated)
 * holds the partial sums and a second kernel reduces them into Y.
 */
typedef struct qa_w4a16_args {
  const void* x;
  const int32_t* qweight;
  const void* scales;
  void* y;
  float* workspace; /* required when the resolved split count is > 1 */
  int64_t x_stride;
  int64_t y_stride;
  int32_t M, N, K;
  int32_t splits; /* 0 = automatic */
  uint32_t* counters; /* optional: (N/128) * ceil(M/16) zeroed counters; with them a split-K
                         call finishes in one launch (the last CTA of each tile adds the
                         partials) and leaves them zero; calls that overlap on the GPU
                         must not share them. NULL: a second kernel adds the partials. */
} qa_w4a16_args;

QA_API int qa_w4a16_gemm(const qa_w4a16_args* args, void* stream);

/*
 * qa_w4a16_gemm without any device allocation, for callers that cannot call
 * cudaMalloc on their hot path (a host framework that only hands out buffers it
 * owns, or a serving loop where an allocation's implicit device synchronisation
 * would stall other streams). No counterpart in the reference.
 * The split-K partial sums go to a fixed 16 MiB array inside the library
 * (4 Mi floats); every GPU that loads the library holds that array until the
 * process exits. The split count is first clamped as in qa_w4a16_gemm (at most
 * K/128, no empty split). With splits = 0 (automatic) a count whose partials
 * (splits * M * N floats) would not fit steps down to the largest that does,
 * down to 1, which needs no scratch; an explicit split count that does not fit
 * returns QA_ERR_INVALID.
 * `workspace` in args is ignored. The first call on each device looks up the
 * array's device address (make that first call before any stream capture).
 * All calls share the array: calls that overlap on the GPU (other streams,
 * other threads) race on it and must be serialised by the caller.
 * Calls no cudaMalloc / cudaFree and no allocating library routine.
 */
QA_API int qa_w4a16_gemm_noalloc(const qa_w4a16_args* args, void* stream);

/* Split count chosen by splits = 0, and the workspace bytes it needs. */
QA_API int qa_w4a16_plan(int32_t M, int32_t N, int32_t K, int32_t* splits, int64_t* workspace_bytes);

/* W'[K, N] (fp16, row-major) = fp16((q - 8) * scale): the dequantisation alone. */
QA_API int qa_w4a16_dequant(const int32_t* qweight, const void* scales, void* out, int32_t K, int32_t N,
                            void* stream);

/*
 * Elementwise steps of the W4A16 verify step (bench config C5; the Llama
 * decoder-layer code the reference runs around its attention,
 * scripts/w4a16_e2e.py:1393-1431). fp16 tensors, fp32 arithmetic, 16-byte
 * aligned, contiguous rows.
 *
 * qa_add_rmsnorm: for each of M rows of `hidden` elements: h += delta (when
 * delta is not NULL, h updated in place), out = fp16(h * rsqrt(mean(h^2) + eps))
 * * w (HF LlamaRMSNorm order).
 */
QA_API int qa_add_rmsnorm(void* h, const void* delta, const void* w, void* out, int32_t M, int32_t hidden,
                          float eps, void* stream);

/*
 * qa_rope_qkv: qkv = [M, (hq + 2 hkv) * head_dim] fused projection of M tokens
 * (n_per_seq tokens per sequence, sequence b = row / n_per_seq). Rotate-half
 * RoPE at position pos[row] with frequencies inv_freq[head_dim/2] (fp32) is
 * applied to the q heads in place; the rotated k heads and the v heads are
 * written to k_cache / v_cache ([B, hkv, S, head_dim] with element strides
 * kv_stride_b, kv_stride_h; token offset kv_offset + row % n_per_seq).
 */
QA_API int qa_rope_qkv(void* qkv, const int32_t* pos, const float* inv_freq, void* k_cache, void* v_cache,
                       int32_t M, int32_t n_per_seq, int32_t hq, int32_t hkv, int32_t head_dim,
                       int64_t kv_stride_b, int64_t kv_stride_h, int32_t kv_offset, void* stream);

/* qa_silu_mul: out[M, F] = silu(gate_up[:, :F]) * gate_up[:, F:] (F % 8 == 0). */
QA_API int qa_silu_mul(const void* gate_up, void* out, int32_t M, int32_t F, void* stream);

/*
 * Reads and clears the device error flag that the tensor-core kernels set when
 * one of their bounded pipeline waits times out (a kernel that hits it stops,
 * frees its resources and leaves its outputs incomplete). Synchronising call.
 * *flag = 0 means no kernel has reported an error since the last call; bit 4
 * means a plan check of the ancestor kernel failed (see qa_ancestor_diagnostics).
 */
QA_API int qa_check_device_error(int* flag);

/*
 * Test hook (no counterpart in the reference): the number of polls after which
 * a pipeline wait of the prefix pass gives up in launches made from now on
 * (0 restores the default, about a second). A small value makes the waits run
 * out on purpose, so that a test can see the abort path end the launch, report
 * through qa_check_device_error, and leave the context usable. The waits that
 * drain a stopping kernel's own copies and MMAs keep the default limit.
 */
QA_API int qa_set_pipeline_wait_limit(uint32_t polls);

/*
 * Diagnostics of the tensor-core ancestor kernel (no counterpart in the
 * reference, whose kernels do not check their index arithmetic): before it
 * stages a tile, the kernel checks that every query row, staged K/V row and key
 * slot of the tile's plan lies inside its sequence; a tile that fails is skipped
 * (its outputs are not written) and the first failure is recorded. out8 (may be
 * NULL) receives [check 1..4 or 0, tile, sequence, value, plan from table,
 * sequence length, tile rows, staged rows]; the record is cleared. Synchronising.
 */
QA_API int qa_ancestor_diagnostics(int32_t* out8);

/* Human-readable name of a status code (static storage). */
QA_API const char* qa_status_string(int status);

/* Library version, e.g. "qattn-b200 0.1.0 sm_100a". */
QA_API const char* qa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* QATTN_B200_H */
