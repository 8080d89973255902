/*
 * tinyserve-b200 C ABI: quantized MoE expert hot path on B200 (sm_100a).
 *
 * All pointers are device pointers owned by the caller unless stated
 * otherwise; `stream` is a cudaStream_t passed as void*.  Every function
 * returns TSB_OK (0) or an error code and never aborts; the message of the
 * last error on the calling thread is available from tsb_last_error().
 * Kernels never allocate: scratch space is the caller's `workspace`.
 *
 * Reference interfaces replaced (tinyserve, file:line):
 *   tsb_quant_matvec  <- torch.ops.tinyserve_ggml.ggml_mul_mat_vec
 *                        (tinyserve/csrc/ggml_ops.cu:461-574) and the MXFP4
 *                        batch-1 vecmat dot_scaled_vecmat
 *                        (tinyserve/triton_dot_scaled.py:68-122)
 *   tsb_dequant       <- gguf_dequant_torch.dequant_tensor
 *                        (tinyserve/gguf_dequant_torch.py:35-78) and
 *                        mxfp4.dequant_mxfp4_no_transpose (tinyserve/mxfp4.py:20-44)
 *   tsb_moe_decode    <- the per-token expert loop of
 *                        ExpertPipeline.execute_layer_experts[_native]
 *                        (tinyserve/expert_pipeline.py:140-164,241-285) with
 *                        GGMLExpertForward / the MXFP4 inline forward
 *                        (tinyserve/ggml_forward.py:68-115,
 *                        tinyserve/expert_forward.py:197-246) and the router
 *                        (tinyserve/_model_hooks.py:466-473); one call per layer.
 */
#ifndef TSB_MOE_H
#define TSB_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define TSB_OK 0
#define TSB_ERR_INVALID 1     /* bad argument (shape, alignment, null pointer) */
#define TSB_ERR_UNSUPPORTED 2 /* format / layout / size not supported */
#define TSB_ERR_CUDA 3        /* a CUDA runtime call failed */
#define TSB_ERR_WORKSPACE 4   /* workspace too small */
#define TSB_ERR_DEVICE 5      /* a kernel reported an error (see tsb_read_device_error) */

/* weight formats: GGUF type ids (tinyserve/gguf_reader.py:15-29) + MXFP4 */
#define TSB_FMT_Q8_0 8
#define TSB_FMT_Q4_K 12
#define TSB_FMT_Q5_K 13
#define TSB_FMT_Q6_K 14
#define TSB_FMT_MXFP4 39 /* no ggml id in the reference; HF *_blocks / *_scales */
/* dense experts (GGUF ids of the float types): plain [rows, cols] tensors,
 * layer entry points only (tsb_moe_decode / tsb_moe_prefill and their
 * workspace functions); tinyserve/expert_forward.py:109-194 */
#define TSB_FMT_F32 0
#define TSB_FMT_F16 1
#define TSB_FMT_BF16 30

/* element types of activations / outputs */
#define TSB_DT_F32 0
#define TSB_DT_BF16 1
#define TSB_DT_F16 2

/* gate/up arrangement */
#define TSB_GU_SEPARATE 0    /* gate [I,H] and up [I,H] (GGUF stores, ggml_forward.py:103-110) */
#define TSB_GU_INTERLEAVED 1 /* gate_up [2I,H]: row 2j = gate j, 2j+1 = up j (expert_forward.py:239-240) */
#define TSB_GU_CHUNKED 2     /* gate_up [2I,H]: rows [0,I) gate, [I,2I) up (expert_forward.py:171-172) */

/* TsbMoeSpec.transposed bits (dense formats only): the projection is stored
 * [in, out] instead of [out, in] and read in place (the reference transposes
 * such weights before F.linear, tinyserve/expert_forward.py:140-149) */
#define TSB_T_GATE_UP 1 /* gate_up [H, 2I] (separate: gate and up [H, I]) */
#define TSB_T_DOWN 2    /* down [I, H] */

/* activation between up and down */
#define TSB_ACT_SILU 0       /* silu(gate) * up (ggml_forward.py:112) */
#define TSB_ACT_SWIGLU_OAI 1 /* clamp-SwiGLU (expert_forward.py:185-187) */

typedef struct {
  int32_t fmt_gate_up; /* format of gate and up projections */
  int32_t fmt_down;    /* format of the down projection */
  int32_t hidden;      /* H */
  int32_t inter;       /* I */
  int32_t n_experts;   /* E */
  int32_t top_k;       /* 1..8 */
  int32_t gate_up_layout; /* TSB_GU_* */
  int32_t activation;  /* TSB_ACT_* */
  float limit;         /* SwiGLU clamp (7.0 for GPT-OSS) */
  float alpha;         /* SwiGLU sigmoid slope (1.702 for GPT-OSS) */
  int32_t out_f32;     /* 0: layer output `out` is bf16 [T, H]; 1: fp32 [T, H] (the
                          unrounded combine, for callers that keep the residual stream
                          in fp32 and for exact parity checks) */
  int32_t transposed;  /* TSB_T_* bits; 0 for quantised formats */
} TsbMoeSpec;

/* One expert's weights (device pointers).  Weights are raw GGUF block streams
 * (row-major flat stream, tinyserve/gguf_dequant_torch.py:72-78) or MXFP4
 * nibble blocks [rows, cols/32, 16] with E8M0 scales [rows, cols/32]. */
typedef struct {
  const void* gate;        /* gate [I,H], or gate_up [2I,H] for interleaved/chunked */
  const void* up;          /* up [I,H] for TSB_GU_SEPARATE, else NULL */
  const void* down;        /* down [H,I] */
  const void* gate_scales; /* MXFP4 scales of gate / gate_up, else NULL */
  const void* up_scales;   /* MXFP4 scales of up, else NULL */
  const void* down_scales; /* MXFP4 scales of down, else NULL */
  const float* gate_bias;  /* optional fp32 [I] */
  const float* up_bias;    /* optional fp32 [I] */
  const float* down_bias;  /* optional fp32 [H] */
} TsbExpert;

/* library version (major*10000 + minor*100 + patch) */
int tsb_version(void);

/* copy the calling thread's last error message into buf; returns its length */
int tsb_last_error(char* buf, size_t n);

/* block geometry of a format: elements and bytes per block */
int tsb_format_info(int fmt, int32_t* block_elems, int32_t* block_bytes);

/* bytes of a [rows, cols] weight: nibble/block stream and (MXFP4) scales */
int tsb_weight_bytes(int fmt, int64_t rows, int64_t cols, int64_t* data_bytes, int64_t* scale_bytes);

/* Bit-exact dequantisation of a [rows, cols] weight into out (fp32 or bf16),
 * identical to dequant_tensor / dequant_mxfp4_no_transpose. */
int tsb_dequant(int fmt, const void* w, const void* scales, int64_t rows, int64_t cols, void* out,
                int out_dtype, void* stream);

/* y[v, :N] = W[N, K] @ x[v, :K] for v < nvec (nvec <= 8 per call is fastest;
 * larger nvec is processed in groups).  x rows are x_stride elements apart,
 * y rows y_stride apart.  W: 16-byte aligned.  K % 32 == 0 (Q8_0, MXFP4) or
 * K % 32 == 0 and N*K % 256 == 0 (K-quants).  dev_err (may be NULL): device
 * int32 the kernel sets non-zero if a bounded wait timed out. */
int tsb_quant_matvec(int fmt, const void* w, const void* scales, int64_t N, int64_t K, const void* x,
                     int x_dtype, int64_t nvec, int64_t x_stride, void* y, int y_dtype, int64_t y_stride,
                     int32_t* dev_err, void* stream);

/* workspace bytes tsb_moe_decode needs for T tokens */
size_t tsb_moe_decode_workspace(const TsbMoeSpec* spec, int32_t T);

/* Dense experts (fmt_gate_up and fmt_down both TSB_FMT_F32 / F16 / BF16, any
 * mix of the three; replaces the dense inline forward
 * tinyserve/expert_forward.py:109-194 and the C++ expert loop
 * tinyserve/csrc/expert_loop.cpp:41-123): tsb_moe_decode and tsb_moe_prefill
 * run every (token, slot) pair of a call in one launch per projection with
 * fp32 accumulation, weights in either orientation (spec->transposed), each
 * weight pointer 16-byte aligned (an unaligned one is reported through the
 * device error word, code 3, and skipped).  Workspace from
 * tsb_moe_decode_workspace for any T. */

/* One MoE layer for T tokens.  T = 1: router + fused gate/up + fused down
 * (three PDL-chained launches).  Several requests decoding together
 * (ExpertBatcher.batch_execute, tinyserve/expert_batcher.py:31-85): up to 16
 * tokens run the T = 1 kernels token by token; more take the grouped path of
 * tsb_moe_prefill, so each routed expert's weights are read once for all its
 * tokens.  tsb_moe_decode_workspace(spec, T) gives the size for either.
 *   experts   device array of n_experts TsbExpert
 *   x         bf16 [T, H]
 *   router_w  bf16 [E, H] (NULL: ids/weights are inputs)
 *   router_b  fp32 [E] or NULL
 *   ids       int32 [T, top_k]  (output if router_w != NULL, else input; as
 *             an input, a negative id marks a slot this call skips, e.g. an
 *             expert another rank owns, and an id >= n_experts is an error
 *             reported through the device error word)
 *   weights   fp32  [T, top_k]  (same)
 *   out       [T, H] = sum_k weights[t,k] * expert_{ids[t,k]}(x[t]), bf16, or
 *             fp32 when spec->out_f32 is set */
int tsb_moe_decode(const TsbMoeSpec* spec, const TsbExpert* experts, const void* x, int32_t T,
                   const void* router_w, const float* router_b, int32_t* ids, float* weights, void* out,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Router alone: logits = bf16(x @ router_w^T + router_b), top-k (ties to the
 * lower id, NaN lowest), softmax over the k selected logits
 * (tinyserve/_model_hooks.py:466-473).  Uses spec->hidden, n_experts, top_k.
 * ids int32 [T, top_k], weights fp32 [T, top_k].  For callers that route
 * before dispatching tokens (expert parallelism). */
int tsb_moe_route(const TsbMoeSpec* spec, const void* x, int32_t T, const void* router_w, const float* router_b,
                  int32_t* ids, float* weights, void* stream);

/* workspace bytes tsb_moe_prefill needs for T tokens (holds the permuted
 * token tiles, the expert weights decoded to fp16 tiles for every expert, the
 * activation tiles and fp32 expert outputs) */
size_t tsb_moe_prefill_workspace(const TsbMoeSpec* spec, int32_t T);

/* One MoE layer for T >= 1 tokens as grouped GEMMs on the tensor cores
 * (replaces ExpertPipeline.execute_layer_experts_batched,
 * tinyserve/expert_pipeline.py:166-239, and group_tokens_by_expert,
 * tinyserve/_fast_cache.pyx:60-85).  Same arguments and routing rule as
 * tsb_moe_decode.  Tokens are grouped by expert on the GPU in (token, slot)
 * order; products run in fp16 with fp32 accumulation (token rows are scaled by
 * exact powers of two to use the fp16 range; weights and the intermediate
 * activations must lie within it). */
int tsb_moe_prefill(const TsbMoeSpec* spec, const TsbExpert* experts, const void* x, int32_t T,
                    const void* router_w, const float* router_b, int32_t* ids, float* weights, void* out,
                    void* workspace, size_t workspace_bytes, void* stream);

/* read (and clear) the device error word kept in a tsb_moe_decode workspace;
 * synchronises the stream.  *code = 0 when no kernel reported an error. */
int tsb_read_device_error(void* workspace, int32_t* code, void* stream);

/* tsb_moe_decode without a caller-provided workspace (no counterpart in the
 * reference).  For callers that have no device scratch memory to hand over
 * (for example a host with a fixed memory plan, or a binding that only sees
 * the tensors it passes): the scratch is a 1 MiB array inside the library,
 * which every GPU that loads the library keeps until the process exits.
 * Layers needing more scratch than that (tsb_moe_decode_workspace) are
 * rejected with TSB_ERR_WORKSPACE.  Calls neither cudaMalloc nor cudaFree.
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and keeps it for later calls; after
 * cudaDeviceReset that cached address is stale, so the process must not
 * call this entry point again on that device.  All calls share the one array: calls
 * that overlap on the GPU (other streams, other threads) race and must be
 * serialised by the caller.  Kernel-side errors of this variant are not
 * reported (there is no workspace to read them from). */
int tsb_moe_decode_noalloc(const TsbMoeSpec* spec, const TsbExpert* experts, const void* x, int32_t T,
                           const void* router_w, const float* router_b, int32_t* ids, float* weights, void* out,
                           void* stream);

/* ---- decode-packed experts (batch-1 decode of Q4_K and MXFP4 layers) -----
 * A one-time repack of all E experts' gate/up/down streams into units of 16
 * rows x 256 columns in the order the decode kernel's tensor-core fragments
 * read them (Q4_K: rows grouped by superblock phase so every unit is one
 * source superblock per row, scales widened to bytes, ~1.03x the Q4_K bytes
 * plus the superblocks that straddle two rows; MXFP4: exactly the MXFP4
 * bytes).  Replaces, for HBM-resident layers, the per-call GGUF decode of
 * ggml_mul_mat_vec (tinyserve/ggml_forward.py:40-62) and the MXFP4 vecmat
 * dot_scaled_vecmat (tinyserve/triton_dot_scaled.py:68-122) inside
 * ExpertPipeline.execute_layer_experts (tinyserve/expert_pipeline.py:140-164);
 * results equal tsb_moe_decode's within the fp32 summation order.
 * tsb_moe_packed_bytes: size of the packed copy, 0 when the spec has no packed
 *   form (needs Q4_K gate/up and down, or MXFP4 gate/up and down; H and I
 *   multiples of 32 and at most 16384; top_k <= 8).
 * tsb_moe_pack: writes it (experts: device array of E TsbExpert, as for
 *   tsb_moe_decode); run once per weight set; returns after the row maps are
 *   on the device (the repack itself is stream-ordered).
 * tsb_moe_decode_packed: tsb_moe_decode's contract (T tokens, optional router,
 *   ids/weights in or out, bf16 or fp32 output) on the packed copy: one
 *   cooperative launch per token (routing, gate/up, activation, down,
 *   combine); `experts` supplies the biases (and the raw streams for T > 16,
 *   which take the grouped path).  Workspace from
 *   tsb_moe_decode_packed_workspace, zero-initialised once; after a non-zero
 *   device error (tsb_read_device_error) zero it again. */
size_t tsb_moe_packed_bytes(const TsbMoeSpec* spec);
int tsb_moe_pack(const TsbMoeSpec* spec, const TsbExpert* experts, void* packed, size_t packed_bytes, void* stream);
size_t tsb_moe_decode_packed_workspace(const TsbMoeSpec* spec, int32_t T);
int tsb_moe_decode_packed(const TsbMoeSpec* spec, const void* packed, const TsbExpert* experts, const void* x,
                          int32_t T, const void* router_w, const float* router_b, int32_t* ids, float* weights,
                          void* out, void* workspace, size_t workspace_bytes, void* stream);

/* Expert-parallel decode over NCCL (the multi-GPU form of one
 * tsb_moe_decode call; the reference runs all experts of a layer on one GPU,
 * tinyserve/expert_pipeline.py:140-164).  The n_experts * world experts of
 * the layer are split evenly: rank r holds experts [r * n, (r + 1) * n), n =
 * local_spec->n_experts, in local_experts (and, optionally, their
 * tsb_moe_pack copy in `packed`, else NULL).  Every rank of the communicator
 * calls it with the same T and passes its own tokens x (bf16 [T, H]) and their
 * routing over the GLOBAL expert ids (ids int32 [T, top_k], weights fp32, e.g.
 * from tsb_moe_route).  On `stream`, with no host synchronisation:
 * all-gather of the tokens and routing, this rank's experts over all world*T
 * rows (other ranks' (token, slot) pairs skipped), reduce-scatter (sum) of the
 * fp32 partial outputs; out [T, H] receives this rank's rows (bf16, or fp32
 * when local_spec->out_f32 is set).
 *   nccl_comm  the caller's ncclComm_t (rank, world as in it); NCCL is found
 *              at run time (libnccl.so.2 already loaded by the process, else
 *              loaded by name); TSB_ERR_UNSUPPORTED when it is absent.
 *   workspace  tsb_ep_decode_workspace(local_spec, T, world, packed != NULL)
 *              bytes, 256-byte aligned, zero-initialised once and used with
 *              the same T on every call (re-zero it before changing T);
 *              tsb_read_device_error(workspace, ...) reads its error word. */
size_t tsb_ep_decode_workspace(const TsbMoeSpec* local_spec, int32_t T, int32_t world, int32_t packed);
int tsb_ep_moe_decode(const TsbMoeSpec* local_spec, const TsbExpert* local_experts, const void* packed,
                      const void* x, int32_t T, const int32_t* ids, const float* weights, void* out,
                      void* nccl_comm, int32_t rank, int32_t world, void* workspace, size_t workspace_bytes,
                      void* stream);

/* The same exchange around tsb_moe_prefill (grouped tensor-core GEMMs over
 * all world*T gathered rows, the multi-GPU form of
 * ExpertPipeline.execute_layer_experts_batched,
 * tinyserve/expert_pipeline.py:166-239), for prefill-sized T (the same on
 * every rank).  Workspace: tsb_ep_prefill_workspace(local_spec, T, world),
 * 256-byte aligned; tsb_read_device_error(workspace, ...) reads its error
 * word. */
size_t tsb_ep_prefill_workspace(const TsbMoeSpec* local_spec, int32_t T, int32_t world);
int tsb_ep_moe_prefill(const TsbMoeSpec* local_spec, const TsbExpert* local_experts, const void* x, int32_t T,
                       const int32_t* ids, const float* weights, void* out, void* nccl_comm, int32_t rank,
                       int32_t world, void* workspace, size_t workspace_bytes, void* stream);

/* ---- whole-model decode around the expert layers (GPT-OSS) ---------------
 * The caller side of the MoE layer in a batch-1 decode step, as the reference
 * runs it through Hugging Face attention with its StaticKVCache
 * (tinyserve/static_kv_cache.py:28-147: keys/values stored as float8 e4m3 and
 * read back exactly) inside its decode loop (tinyserve/offload.py:219-287).
 *
 * tsb_gqa_decode_attention: one token's grouped-query attention.  qkv is the
 *   bf16 [n_q + 2 n_kv, head_dim] output of the fused q|k|v projection before
 *   RoPE; cos / sin bf16 [max_seq, head_dim / 2] tables (halves rotated); pos a
 *   device int64 holding the token's position (read on the device, so the call
 *   can sit in a CUDA graph).  The new key (roped) and value are stored in the
 *   caches [n_kv, max_seq, head_dim] (e4m3 when cache_fp8, else bf16) at pos;
 *   scores over positions [0, pos] (the last `window` when window > 0) scaled
 *   by `scale`, softmax with the per-query-head sink logit sinks[n_q] in the
 *   denominator, out bf16 [n_q, head_dim].  head_dim must be 64, n_q / n_kv <=
 *   16.  Workspace: tsb_gqa_decode_workspace bytes, 256-byte aligned,
 *   zero-initialised once; one workspace serves successive calls on a stream.
 * tsb_add_rmsnorm: x[r] += delta[r] (fp32 residual rows, delta fp32 or bf16 or
 *   NULL), out[r] = bf16(weight * x[r] / sqrt(mean(x[r]^2) + eps)). */
size_t tsb_gqa_decode_workspace(int32_t n_q_heads, int32_t n_kv_heads, int32_t max_seq);
int tsb_gqa_decode_attention(const void* qkv, int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                             const void* cos, const void* sin, const int64_t* pos, void* k_cache, void* v_cache,
                             int32_t cache_fp8, int32_t max_seq, int32_t window, const float* sinks, float scale,
                             void* out, void* workspace, size_t workspace_bytes, void* stream);
int tsb_add_rmsnorm(float* x, const void* delta, int32_t delta_dtype, const float* weight, float eps, int32_t rows,
                    int32_t hidden, void* out, void* stream);
/* The same attention for `batch` sequences decoding together (several
 * requests served at once, tinyserve/server.py:48-150): row b of qkv / out,
 * position pos[b], cache slot slots[b] (the caches hold slots slot_stride
 * elements apart, each [n_kv, max_seq, head_dim]).  Workspace from
 * tsb_gqa_decode_batch_workspace for that batch size. */
size_t tsb_gqa_decode_batch_workspace(int32_t n_q_heads, int32_t n_kv_heads, int32_t max_seq, int32_t batch);
int tsb_gqa_decode_attention_batch(const void* qkv, int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                                   const void* cos, const void* sin, const int64_t* pos, const int32_t* slots,
                                   int64_t slot_stride, void* k_cache, void* v_cache, int32_t cache_fp8,
                                   int32_t max_seq, int32_t window, const float* sinks, float scale, void* out,
                                   int32_t batch, void* workspace, size_t workspace_bytes, void* stream);
/* RMSNorm + fused q|k|v projection + tsb_gqa_decode_attention in one launch
 * (thread-block clusters of 8 or 16 CTAs per KV head exchange the head
 * group's projections through distributed shared memory): x_in / delta /
 * x_out / norm_weight as tsb_norm_gemv_bf16, weight / bias the bf16 q|k|v
 * projection [(n_q + 2 n_kv) * head_dim, hidden] (16-byte aligned), the rest
 * as tsb_gqa_decode_attention; no workspace.  TSB_ERR_UNSUPPORTED when the
 * shape does not fit the kernel's shared memory (callers then use the two
 * separate entry points). */
int tsb_norm_qkv_attention(const float* x_in, const float* delta, float* x_out, const float* norm_weight, float eps,
                           const void* weight, const void* bias, int32_t hidden, int32_t n_q_heads,
                           int32_t n_kv_heads, int32_t head_dim, const void* cos, const void* sin,
                           const int64_t* pos, void* k_cache, void* v_cache, int32_t cache_fp8, int32_t max_seq,
                           int32_t window, const float* sinks, float scale, void* out, void* stream);
/* y = bf16(W x + bias): one bf16 [N, K] weight (16-byte aligned, K % 8 == 0,
 * K <= 16384), bf16 x [K], optional bf16 bias [N], bf16 y [N]; the batch-1
 * attention projections of the decode step (nn.Linear in the reference's
 * model). */
int tsb_gemv_bf16(const void* weight, const void* bias, int32_t N, int32_t K, const void* x, void* y, void* stream);
/* The same GEMV with the sublayer's RMSNorm in front: x = bf16(norm_weight *
 * RMSNorm(x_in + delta)) (x_in fp32 [K], delta fp32 [K] or NULL), computed by
 * every CTA; x_in + delta is also stored to x_out (fp32 [K], not aliasing
 * x_in or delta).  y = bf16(W x + bias). */
int tsb_norm_gemv_bf16(const float* x_in, const float* delta, float* x_out, const float* norm_weight, float eps,
                       const void* weight, const void* bias, int32_t N, int32_t K, void* y, void* stream);
/* The same GEMV adding its bf16 result into an fp32 residual (resid[N] +=
 * bf16(W x + bias)); the last CTA then writes h_out = bf16(norm_weight *
 * RMSNorm(resid)) [N].  counter: a device uint32, zero-initialised once
 * (the kernel resets it). */
int tsb_gemv_bf16_residual(const void* weight, const void* bias, int32_t N, int32_t K, const void* x, float* resid,
                           const float* norm_weight, float eps, void* h_out, uint32_t* counter, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TSB_MOE_H */
