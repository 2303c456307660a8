/*
 * koemi_b200.h -- C ABI of libkoemi_b200.so, the sm_100a kernels behind the
 * HERM forward hot path (affine scan, RMSNorm-SiLU, causal surprise with
 * salient admission, MoE route / permute / grouped expert MLP / combine).
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are device pointers to contiguous row-major data
 *     on the device that is current when the call is made.
 *   - `stream` is a cudaStream_t passed as void*; NULL means the legacy
 *     default stream. Every kernel is enqueued on that stream and the call
 *     returns without synchronising.
 *   - Inputs are borrowed, outputs and workspaces are owned by the caller.
 *     The library never frees caller memory and allocates nothing on a
 *     compute call (one small per-device status word is allocated on the
 *     first call that uses a device).
 *   - The return value is KOEMI_OK (0) or a negative KOEMI_ERR_* code; the
 *     message for the calling thread is read with koemi_last_error().
 *   - `dtype` arguments take a koemi_dtype value.
 *
 * Reference interfaces named below are paths inside the Koemi-5HOM project.
 */
#ifndef KOEMI_B200_H
#define KOEMI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KOEMI_ABI_VERSION 1

#if defined(__GNUC__)
#define KOEMI_API __attribute__((visibility("default")))
#else
#define KOEMI_API
#endif

enum koemi_status {
    KOEMI_OK = 0,
    KOEMI_ERR_INVALID = -1,     /* bad shape, dtype, pointer or alignment */
    KOEMI_ERR_CUDA = -2,        /* a CUDA runtime or driver call failed */
    KOEMI_ERR_UNSUPPORTED = -3, /* valid request outside what the kernels cover */
    KOEMI_ERR_TIMEOUT = -4,     /* a bounded device-side wait gave up */
    KOEMI_ERR_WORKSPACE = -5    /* caller workspace smaller than required */
};

typedef enum koemi_dtype {
    KOEMI_F32 = 0,
    KOEMI_F16 = 1,
    KOEMI_BF16 = 2,
    KOEMI_F64 = 3,
    KOEMI_I32 = 4,
    KOEMI_I64 = 5,
    KOEMI_BOOL = 6
} koemi_dtype;

/* ---------------------------------------------------------------- library */

/* Mirrors CUDA_EXTENSION_ABI_VERSION / KOEMI_CUDA_ABI_VERSION
 * (src/koemi/cuda_kernels/loader.py:32, core/rmsnorm_silu.cpp:74,
 * moe/moe_kernels.cpp:257). Returns KOEMI_ABI_VERSION. */
KOEMI_API int koemi_abi_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to `capacity`) and returns its full length. */
KOEMI_API size_t koemi_last_error(char *buffer, size_t capacity);

/* Reads and clears the device-side status word of `device`, written by a
 * bounded wait that gave up (KOEMI_ERR_TIMEOUT) or 0. Synchronises `device`. */
KOEMI_API int koemi_device_status(int device, int *status_out);

/* Allocates the per-device status word and sets kernel attributes for
 * `device` ahead of time. Call once per device before capturing any of
 * these kernels into a CUDA graph; compute calls otherwise do it lazily. */
KOEMI_API int koemi_device_init(int device);

/* ------------------------------------------------------------- sampling */

/* Greedy decode tokens: out[r] = argmax over c of logits[r * row_stride + c]
 * with column pad_id scored as -inf (pass -1 for no mask), ties to the first
 * index and NaN ranked above every number, as torch.argmax does on the
 * masked row. logits fp32 [rows, vocab] (row stride in elements), out int64
 * [rows]. Replaces the greedy path of TokenSampler
 * (src/koemi/runtime/fast_decode.py:40-87). */
KOEMI_API int koemi_sampler_greedy(const float *logits, int64_t rows, int64_t vocab, int64_t row_stride,
                                   int64_t pad_id, int64_t *out, void *stream);

/* Temperature sampling of one token per row from softmax(logits / T), PAD
 * (pad_id) excluded, as a counter-based Gumbel-max: out[r] = argmax_v of
 * logit_v / T - log(-log(u_v)), u_v drawn from (seed, stream_offset + r,
 * *step, v) by SplitMix64 (the formula is in sampler.cu; the oracle restates
 * it bit for bit), so each stream's draws are its own and reproducible.
 * `step` is a device int64 the caller advances between calls (graph
 * capturable). `thresholds` (fp32 [rows], may be NULL) drops logits below the
 * row's value (the top-k filter of the reference). NaN logits are never
 * chosen. Replaces TokenSampler's sampled path (runtime/fast_decode.py:72-80:
 * softmax(scores / T) then torch.multinomial with a generator): the same
 * distribution from a different random stream. */
KOEMI_API int koemi_sampler_temperature(const float *logits, int64_t rows, int64_t vocab, int64_t row_stride,
                                        int64_t pad_id, float temperature, uint64_t seed, int64_t stream_offset,
                                        const int64_t *step, const float *thresholds, int64_t *out, void *stream);

/* ------------------------------------------------------------ dense front */

/* Affine recurrent scan h_t = a_t * h_{t-1} + b_t over [batch, length,
 * features], carried from `initial` ([batch, features]; NULL = zeros).
 * `retention` is [batch, length, features], or [batch, length] when
 * `broadcast_retention` is nonzero (one coefficient per position).
 * Accumulates in fp32 (fp64 for KOEMI_F64); `states` gets every h_t in dtype.
 * With a workspace of koemi_dense_affine_scan_workspace() bytes (16-byte
 * aligned) the sequence is split into segments scanned by separate CTAs that
 * pass carries by decoupled look-back; with workspace NULL one CTA walks each
 * (batch row, 32 features) lane group through the whole sequence. Both give
 * the same recurrence in fp32; the association order differs.
 * Replaces dense/affine_scan.cu:119-167 (`forward` behind
 * dense_affine_scan, dense/affine_scan.py:51-82). */
KOEMI_API size_t koemi_dense_affine_scan_workspace(int64_t batch, int64_t length, int64_t features,
                                         int dtype);
KOEMI_API int koemi_dense_affine_scan_forward(const void *retention, const void *increment,
                                    const void *initial, void *states,
                                    int64_t batch, int64_t length, int64_t features,
                                    int broadcast_retention, int dtype, void *workspace,
                                    size_t workspace_bytes, void *stream);

/* Reverse-time adjoint of the scan: grad_increment, grad_retention (full
 * [batch, length, features] even when broadcast; the caller reduces) and
 * grad_initial. Replaces dense/affine_scan.cu:169-226. */
KOEMI_API int koemi_dense_affine_scan_backward(const void *retention, const void *initial,
                                     const void *states, const void *grad_states,
                                     void *grad_retention, void *grad_increment,
                                     void *grad_initial, int64_t batch, int64_t length,
                                     int64_t features, int broadcast_retention, int dtype,
                                     void *stream);

/* Gate epilogue of BoundedRecurrentState.gates (model/memory.py:22-26) with
 * the padding masks of network.py:308-309, fused with the T==1 scan step:
 * a = lo + (hi - lo) * sigmoid(pre_a), b = (1 - a) * tanh(pre_c);
 * padding rows get a = 1, b = 0. `projections` is [rows, 2*features] fp32
 * (pre_a | pre_c). Writes retention/increment (fp32, [rows, features]). */
KOEMI_API int koemi_dense_bounded_gates(const float *projections, const uint8_t *valid,
                              float *retention, float *increment, int64_t rows,
                              int64_t features, float minimum_retention,
                              float maximum_retention, void *stream);

/* Decode step of the gates and the scan (one token per stream), in place:
 * a = lo + (hi - lo) sigmoid(pre_a), b = (1 - a) tanh(pre_c) (a = 1, b = 0 where
 * !valid); prior_out <- working (cast to prior_dtype, may be NULL);
 * working <- a * working + b; h_out[row * h_stride + f] <- the new working
 * (in prior_dtype, may be NULL); h_copy[row * features + f] <- the same value
 * again (may be NULL: the decode step's rows of the next head pass).
 * `projections` is [batch, 2*features] fp32 (pre_a | pre_c). Fuses
 * BoundedRecurrentState.gates (model/memory.py:22-26), the masks of
 * network.py:308-309 and the T == 1 affine scan (model/scan.py:17-30). */
KOEMI_API int koemi_dense_decode_step(const float *projections, const uint8_t *valid, float *working,
                            void *prior_out, void *h_out, int64_t h_stride, void *h_copy, int64_t batch,
                            int64_t features, float minimum_retention, float maximum_retention,
                            int prior_dtype, void *stream);

/* Associative memory over a window of `length` positions (prefill), in place:
 * for t = 0..length-1 of every stream, den = n . q_t, reg = den + 2^-8,
 * read_t[i] = (den / reg) (basis[i] . q_t) / reg, then
 * basis[i] = decay_t basis[i] + write_t value_t[i] f_t and
 * n = decay_t n + write_t f_t. decay, write fp32 [batch, length]; value,
 * read_out fp32 [batch, length, width]; features, query_features fp32
 * [batch, length, feature_count]; basis fp32 [batch, width, feature_count]
 * (16-byte aligned), normaliser fp32 [batch, feature_count]. feature_count
 * must be 4, 8, 16 or 32 (other counts up to 32 run zero-padded to the next
 * of these: a zero feature never writes nor reads). Replaces the window read of
 * HierarchicalAssociativeMemory.scan_and_read (model/memory.py:97-144,146-242). */
KOEMI_API int koemi_assoc_window_scan_read(const float *decay, const float *write, const float *value,
                                           const float *features, const float *query_features, float *basis,
                                           float *normalizer, float *read_out, int64_t batch, int64_t length,
                                           int64_t width, int64_t feature_count, void *stream);

/* Dense projection out = a W^T + bias on tcgen05 tensor cores, fp32 output:
 * a [rows, k] (row stride a_stride elements, bf16/f16), W [n, k] (same dtype,
 * contiguous), bias [n] (same dtype, may be NULL), out fp32 rows of
 * out_stride. Small row counts split K across CTAs and reduce the fp32
 * partials in a fixed order (deterministic) through `workspace` of
 * koemi_dense_projection_workspace() bytes. The projections of the HERM block
 * (gates, local, associative, fusion, head; network.py:97,106, memory.py:17-18,
 * 70-75,294-295) use it at decode. k and a_stride must be multiples of 8. */
KOEMI_API size_t koemi_dense_projection_workspace(int64_t rows, int64_t n, int64_t k, int dtype);
KOEMI_API int koemi_dense_projection(const void *a, int64_t a_stride, const void *weight, const void *bias,
                           float *out, int64_t out_stride, int64_t rows, int64_t n, int64_t k, int dtype,
                           void *workspace, size_t workspace_bytes, void *stream);
/* The same projection for weights that no work still in flight on `stream`
 * writes (model parameters): the kernel is launched with programmatic stream
 * serialization and loads its first weight tiles while the previous kernel of
 * the stream finishes, reading `a` (and the bias) only after that kernel has
 * completed. Same arguments, results and limits as koemi_dense_projection;
 * the decode step's block projections use it (same reference lines). */
KOEMI_API int koemi_dense_projection_resident(const void *a, int64_t a_stride, const void *weight, const void *bias,
                           float *out, int64_t out_stride, int64_t rows, int64_t n, int64_t k, int dtype,
                           void *workspace, size_t workspace_bytes, void *stream);

/* A batch of small products on tcgen05 tensor cores, fp32 output:
 * out[g * M + i, j] = sum_k A[g * M + i, k] B[g * N + j, k] for every group
 * g < groups (M = rows_per_group), A [groups * M, k] and B [groups * N, k]
 * bf16/f16 row-major, out fp32 [groups * M, N]. The prefill's ring reads use
 * it per stream: the [C, L + C] scores (queries x ring keys) and the weighted
 * sums (weights x transposed ring values) of LocalKeyValueMemory.read_window
 * and the salient read (model/memory.py:332-361, 405-429). k a multiple of 8. */
KOEMI_API int koemi_grouped_projection(const void *a, const void *b, float *out, int64_t groups,
                                       int64_t rows_per_group, int64_t n, int64_t k, int dtype, void *stream);

/* Row blocks converted to `dtype` (F32/BF16/F16) and packed side by side:
 * out[r, o_p + j] = sources[p][r * strides[p] + j] for j < widths[p], where
 * o_p = widths[0] + ... + widths[p-1], for rows r < rows and 1 to 8 parts
 * (fp32 sources; widths and out_stride multiples of 4, strides even; source
 * rows 16-byte aligned, 8 where the stride is not a multiple of 4; `sources`,
 * `strides`, `widths` are host arrays). The window path
 * builds the fusion input [h | memory | local | salient] (network.py:723-732)
 * and the prior [state ; h[:-1]] (network.py:320-325) with it in the GEMMs'
 * operand type, one read of each fp32 element. */
KOEMI_API int koemi_window_pack_rows(const float *const *sources, const int64_t *strides, const int64_t *widths,
                                     int parts, int64_t rows, void *out, int64_t out_stride, int dtype, void *stream);

/* The slot operands of a window ring read (LocalKeyValueMemory.read_window
 * and the salient read, model/memory.py:332-361, 405-429): for every stream b
 * the slots [carried ring (carried rows) ; window (length rows)] padded with
 * zero slots to `padded` (a multiple of 8, >= carried + length), as stacked
 * keys keys_out [batch, padded, width] and transposed values values_t_out
 * [batch, width, padded] in `dtype` (F32/BF16/F16). Inputs are fp32 with
 * contiguous rows of `width` (a multiple of 4): carried keys/values at batch
 * stride carried_stride, window keys/values at batch stride window_stride.
 * These are the B operands of koemi_grouped_projection for the scores and
 * the weighted sum. */
KOEMI_API int koemi_window_slot_operands(const float *carried_keys, const float *carried_values,
                                         int64_t carried_stride, int64_t carried, const float *keys,
                                         const float *values, int64_t window_stride, int64_t length, int64_t batch,
                                         int64_t width, int64_t padded, void *keys_out, void *values_t_out, int dtype,
                                         void *stream);

/* ------------------------------------------------------------- core front */

/* y = silu(x * rsqrt(mean(x^2) + eps) * w), inv_rms[row] = rsqrt(...).
 * x, w, y in dtype (F32/F16/BF16); inv_rms fp32 [rows].
 * Replaces core/rmsnorm_silu.cu:63-91,148-217 (fused_rmsnorm_silu,
 * core/rmsnorm_silu.py:37-42). */
KOEMI_API int koemi_core_rmsnorm_silu_forward(const void *x, const void *weight, void *y,
                                    float *inv_rms, int64_t rows, int64_t hidden, float eps,
                                    int dtype, void *stream);

/* Backward of the above: grad_x in dtype, grad_weight fp32 [hidden]
 * (overwritten, deterministic two-stage reduction through `workspace` of
 * koemi_core_rmsnorm_silu_backward_workspace() bytes).
 * Replaces core/rmsnorm_silu.cu:94-132. */
KOEMI_API size_t koemi_core_rmsnorm_silu_backward_workspace(int64_t rows, int64_t hidden);
KOEMI_API int koemi_core_rmsnorm_silu_backward(const void *grad_y, const void *x, const void *weight,
                                     const float *inv_rms, void *grad_x, float *grad_weight,
                                     int64_t rows, int64_t hidden, void *workspace,
                                     size_t workspace_bytes, int dtype, void *stream);

/* Gated form y = silu(gate) * (x * rsqrt(mean(x^2) + eps) * w): the config-3
 * variant of the fused norm (no reference kernel; restated from
 * RootMeanSquareNorm, model/layers.py:14-16, and F.silu). */
KOEMI_API int koemi_core_gated_rmsnorm_silu_forward(const void *x, const void *gate, const void *weight,
                                          void *y, float *inv_rms, int64_t rows,
                                          int64_t hidden, float eps, int dtype, void *stream);

/* Plain RMSNorm with optional residual and row select, the three norms of the
 * block (network.py:86,98; experts.py:127,204-205):
 *   v = x + residual (residual may be NULL);
 *   y = v * rsqrt(mean(v^2) + eps) * w        where keep[row] (or keep NULL)
 *   y = x                                     where !keep[row].
 * x/residual/y/w share `dtype`; `out_dtype` may differ (cast on store). */
KOEMI_API int koemi_core_rmsnorm_forward(const void *x, const void *residual, const void *weight,
                               const uint8_t *keep, void *y, int64_t rows, int64_t hidden,
                               float eps, int dtype, int out_dtype, void *stream);

/* ------------------------------------------------------------ think front */

/* Causal surprise s = 1 - exp(-NLL / ln(C)) of target_ids under
 * softmax(prior @ weight^T + bias) over C content ids; 0 where !valid.
 * prior [rows, width], weight [C, width], bias [C] share `dtype`; out in
 * `out_dtype` ([rows]). `nll_out` (fp32 [rows], may be NULL) receives the
 * raw NLL. Needs koemi_think_surprise_workspace() bytes of workspace.
 * Replaces think/surprise_kernel.cu:195-215 + 85-134 (causal_surprise,
 * think/surprise.py:91-128) without materialising the [rows, C] logits. */
KOEMI_API size_t koemi_think_surprise_workspace(int64_t rows, int64_t width, int64_t content_vocab,
                                      int dtype);
KOEMI_API int koemi_think_causal_surprise_forward(const void *prior, const void *weight, const void *bias,
                                        const int64_t *target_ids, const uint8_t *valid,
                                        void *out, float *nll_out, int64_t rows, int64_t width,
                                        int64_t content_vocab, int dtype, int out_dtype,
                                        void *workspace, size_t workspace_bytes, void *stream);

/* Backward of the causal surprise: dlogits [rows, content_vocab] fp32 =
 * dL/dNLL_r * (softmax(prior_r W^T + b) - onehot(target_r)), with
 * dL/dNLL_r = grad_r * exp(-NLL_r / ln C) / ln C and zero rows where !valid
 * (valid may be NULL). `nll` is the forward's per-row NLL (nll_out of
 * koemi_think_causal_surprise_forward); grad_surprise has the prior's dtype.
 * The logits are recomputed tile by tile (tcgen05 for bf16/f16, FMA tiles for
 * f32) and never stored; the caller forms dprior = dlogits W,
 * dW = dlogits^T prior and db = column sums (fp32 library GEMMs, as the
 * reference does). Workspace: koemi_think_surprise_backward_workspace(rows).
 * Replaces think/surprise_kernel.cu:137-261 (an fp32 logits at::mm, then
 * the logits-gradient kernel). */
KOEMI_API size_t koemi_think_surprise_backward_workspace(int64_t rows);
KOEMI_API int koemi_think_causal_surprise_backward(const void *prior, const void *weight, const void *bias,
                                                   const int64_t *target_ids, const uint8_t *valid,
                                                   const void *grad_surprise, const float *nll, float *dlogits,
                                                   int64_t rows, int64_t width, int64_t content_vocab, int dtype,
                                                   void *workspace, size_t workspace_bytes, void *stream);

/* Merged head pass of a decode step (one read of the head for two uses):
 * rows [lse_rows + logit_rows, width] (bf16/f16, contiguous) against the full
 * head W [vocab, width] + bias [vocab] on tcgen05 tensor cores.
 *  - rows [0, lse_rows) (the working state of every block after this step,
 *    i.e. the next step's surprise priors): per 256-wide vocabulary slice a
 *    (max, sum exp, -inf) triple of the fp32 logits with column pad_id left
 *    out, into partials [slices][lse_rows][3] (slices =
 *    koemi_think_head_pass_slices(vocab)); the target is not known yet.
 *  - rows [lse_rows, lse_rows + logit_rows) (the final contexts): fp32 logits
 *    [logit_rows, vocab] = row W^T + bias, every column.
 * Replaces the separate content-head surprise pass of the next step and this
 * step's logits head (calculate_surprise and predict_tokens,
 * model/network.py:677-701). */
KOEMI_API int64_t koemi_think_head_pass_slices(int64_t vocab);
KOEMI_API int koemi_think_head_pass(const void *rows, int64_t lse_rows, int64_t logit_rows, int64_t width,
                                    const void *head_weight, const void *head_bias, int64_t vocab, int64_t pad_id,
                                    float *partials, float *logits, int dtype, void *stream);

/* Surprise of the head pass's rows once their targets are known (the next
 * step's tokens): row r (block-major, stream r % batch) gets
 * NLL = logsumexp(partials) - (prior_r . W[token] + b[token]) and
 * s = 1 - exp(-NLL / ln C), C = vocab - 1 (PAD excluded), 0 where !valid.
 * Tokens must lie in [0, vocab) (the sampler's output). fp32 surprise [rows].
 * Same value as causal_surprise (think/surprise.py:91-128) up to the fp32
 * summation order. */
KOEMI_API int koemi_think_surprise_from_partials(const void *prior, const void *head_weight, const void *head_bias,
                                                 const int64_t *token_ids, const uint8_t *valid,
                                                 const float *partials, int64_t slices, int64_t rows, int64_t batch,
                                                 int64_t width, int64_t vocab, int64_t pad_id, int dtype,
                                                 float *surprise, void *stream);

/* Salient admission and ring compaction (network.py:349 and
 * LocalKeyValueMemory.salient_tail, model/memory.py:431-455): admits
 * position t of row b when valid && surprise > threshold, then keeps the
 * latest `capacity` admitted entries of [carried ring ; window] in temporal
 * order, ring slots oldest first and empty slots (zero, invalid) leading.
 * carried_* are [batch, carried, width] / [batch, carried]; keys/values are
 * [batch, length, width]; outputs are [batch, capacity, width] /
 * [batch, capacity] and must not alias the inputs.
 * `admission_out` ([batch, length] bytes, may be NULL) receives the mask. */
KOEMI_API int koemi_think_salient_admission(const float *carried_keys, const float *carried_values,
                                  const uint8_t *carried_valid, const float *keys,
                                  const float *values, const float *surprise,
                                  const uint8_t *valid, float threshold,
                                  float *out_keys, float *out_values, uint8_t *out_valid,
                                  uint8_t *admission_out, int64_t batch, int64_t carried,
                                  int64_t length, int64_t width, int64_t capacity,
                                  void *stream);

/* One decode step of both exact-memory rings of every stream, in place
 * (LocalKeyValueMemory.read_window / read_salient_window / tail /
 * salient_tail, model/memory.py:332-455, and the admission of
 * network.py:349, at sequence length 1). Rings are circular: the local ring's
 * oldest slot is *local_head for every stream; salient ring b holds
 * salient_count[b] admitted entries starting at salient_head[b]. Reads the
 * query rows (queries + b*query_stride, fp32 width), computes the softmax
 * reads of both rings (scale 1/sqrt(width)) and the local novelty, then
 * writes the new entry (entries + b*entry_stride: key | value, zeroed when
 * !valid) over the oldest local slot and, when valid && surprise > threshold,
 * into the salient ring (dropping its oldest entry when full). Outputs go to
 * local_out / salient_out rows of out_stride (out_dtype); novelty_out and admission_out
 * ([batch]) may be NULL. Ring rows are ring_dtype (KOEMI_F32, or KOEMI_BF16 to
 * halve the ring traffic), 16-byte aligned, width a multiple of 4 (fp32) or 8
 * (bf16); arithmetic is fp32. The caller advances *local_head once per step. */
KOEMI_API int koemi_think_ring_decode_step(
    const float *queries, int64_t query_stride, const float *entries, int64_t entry_stride,
    const uint8_t *valid, const float *surprise, float threshold, void *local_keys, void *local_values,
    uint8_t *local_valid, const int64_t *local_head, void *salient_keys, void *salient_values,
    uint8_t *salient_valid, int32_t *salient_head, int32_t *salient_count, void *local_out,
    void *salient_out, int64_t out_stride, float *novelty_out, uint8_t *admission_out, int64_t batch,
    int64_t width, int64_t local_slots, int64_t salient_slots, int ring_dtype, int out_dtype, void *stream);

/* One decode step of the rank-one associative memory, in place
 * (HierarchicalAssociativeMemory.project / read / update with the fast write
 * terms, model/memory.py:82-95,248-255,279-287, network.py:338-347):
 * `projections` rows (stride proj_stride, 8-byte aligned) hold key | query |
 * value_pre | decay_pre | write_pre as produced by one GEMM. The feature
 * logits are either given in feature_logits ([2, batch, features]: key then
 * query logits) or, when it is NULL, computed in the kernel from
 * feature_weight [features, width] and feature_bias ([features] or NULL),
 * both weight_dtype (f32, f16 or bf16), with the key / query rounded to
 * weight_dtype and fp32 accumulation.
 * Writes the confidence-weighted read to read_out rows (stride read_stride, out_dtype)
 * from the memory before this step's write, then basis <- decay * basis +
 * w * tanh(value) f^T and normalizer <- decay * normalizer + w f, with
 * w = sigmoid(write_pre) (0.25 + 0.75 clamp(surprise)) (surprise may be NULL:
 * 0); invalid rows keep their memory. */
KOEMI_API int koemi_assoc_decode_step(const float *projections, int64_t proj_stride,
                            const float *feature_logits, const void *feature_weight, const void *feature_bias,
                            int weight_dtype, const float *surprise, const uint8_t *valid,
                            float *basis, float *normalizer, void *read_out, int64_t read_stride,
                            int64_t batch, int64_t width, int64_t features, int out_dtype, void *stream);

/* -------------------------------------------------------------- moe front */

/* Content-hash top-k routing (model/experts.py:30-38,283-289): assignments
 * [tokens, top_k] int64, -1 for invalid tokens, computed in 64-bit arithmetic
 * exactly as the torch runner does. ids are KOEMI_I32 or KOEMI_I64.
 * Replaces moe/moe_kernels.cu:45-66,352-388 (route_topk_valid,
 * moe/__init__.py:128-176). */
KOEMI_API int koemi_moe_route_topk(const void *token_ids, const void *previous_token_ids,
                         const uint8_t *valid, int64_t *assignments, int64_t tokens,
                         int64_t expert_count, int64_t top_k, int index_dtype, void *stream);

/* Learned top-k gate (LearnedExpertMixture.forward, model/router.py:43-59):
 * probabilities = softmax_fp32(gate_logits) per token, top-k in descending
 * probability (selected on the logits, lowest expert id first among equal
 * values), weights = raw probabilities (renormalize != 0 divides by their
 * sum); invalid tokens get expert -1 / weight 0. gate_logits fp32
 * [tokens, E]; `probabilities` (fp32 [tokens, E], may be NULL) receives the
 * softmax, zeroed on invalid tokens, for the RouterStatistics sums. */
KOEMI_API int koemi_moe_learned_topk(const float *gate_logits, const uint8_t *valid, int64_t *assignments,
                           float *weights, float *probabilities, int64_t tokens,
                           int64_t expert_count, int64_t top_k, int renormalize, void *stream);

/* Stable permutation of token-expert pairs into expert segments
 * (moe/moe_kernels.cu:68-145,390-499; experts.py:171-216,261-267): pair
 * p = token*top_k + slot is valid when valid[token], 0 <= e < E and no earlier
 * slot of that token names the same e; valid pairs are ordered by expert then
 * by p, invalid pairs follow. Outputs: sorted_context [pairs, width] (rows of
 * context, zero past the valid count), sorted_rows [pairs] (token of each
 * sorted pair), sorted_experts [pairs] (E for invalid), segment_offsets
 * [E + 1] (exclusive offsets, last = valid count) and, when non-NULL,
 * pair_positions [pairs] (sorted index of pair p). sorted_context may be NULL
 * to skip the gather. Bit-exact with a stable argsort. */
KOEMI_API size_t koemi_moe_permute_workspace(int64_t tokens, int64_t top_k, int64_t expert_count);
KOEMI_API int koemi_moe_permute_topk(const void *context, const void *assignments, const uint8_t *valid,
                           void *sorted_context, int64_t *sorted_rows, int64_t *sorted_experts,
                           int64_t *segment_offsets, int64_t *pair_positions, int64_t tokens,
                           int64_t width, int64_t top_k, int64_t expert_count, int context_dtype,
                           int assignment_dtype, void *workspace, size_t workspace_bytes,
                           void *stream);

/* Allocation-free variant of koemi_moe_permute_topk, for callers that cannot
 * allocate device memory (a host runtime that only hands over buffers it
 * already owns, or code that must not call cudaMalloc while other work is in
 * flight). It has no counterpart in the reference. Arguments and outputs are
 * those of koemi_moe_permute_topk minus the workspace: the scratch is a fixed
 * 2 MiB device array inside the library, held by every GPU that loads it
 * until the process exits. A request fits when
 * koemi_moe_permute_workspace(tokens, top_k, expert_count) <= 2 MiB: 65536
 * token-expert pairs always fit, at any expert count, and more fit when there
 * are few experts; larger requests fail with KOEMI_ERR_UNSUPPORTED and a
 * message that gives the bytes needed. The first call in a context looks up
 * that array's address with the device current (again after the context
 * changes, e.g. after cudaDeviceReset), so make that first call before any
 * stream capture. All calls share the array: calls that can overlap on the
 * GPU (different streams, different host threads) race and must be
 * serialised by the caller. Allocates nothing. */
KOEMI_API int koemi_moe_permute_topk_static(const void *context, const void *assignments, const uint8_t *valid,
                                  void *sorted_context, int64_t *sorted_rows, int64_t *sorted_experts,
                                  int64_t *segment_offsets, int64_t *pair_positions, int64_t tokens,
                                  int64_t width, int64_t top_k, int64_t expert_count, int context_dtype,
                                  int assignment_dtype, void *stream);

/* Grouped gated expert MLP over sorted segments (GatedFeedForward,
 * model/layers.py:19-29): for sorted pair i of expert e,
 *   y_i = W_o[e] (silu(W_g[e] x_i + b_g[e]) * (W_v[e] x_i + b_v[e])) + b_o[e];
 * rows at or past segment_offsets[E] are zero. Weights: gate/value
 * [E, H, D], biases [E, H], output [E, D, H], output bias [E, D].
 * BF16/F16 run on tcgen05 tensor cores (fp32 accumulate, the gated hidden
 * rounded to dtype between the two contractions); F32 runs an fp32 FMA path.
 * Workspace: koemi_moe_grouped_mlp_workspace() bytes.
 * Replaces moe/moe_kernels.cu:147-199,276-320,501-558
 * (grouped_expert_mlp_inference, moe/__init__.py:231-312). */
KOEMI_API size_t koemi_moe_grouped_mlp_workspace(int64_t pairs, int64_t input_width, int64_t hidden_width,
                                       int64_t expert_count, int dtype);
KOEMI_API int koemi_moe_grouped_expert_mlp(const void *sorted_context, const int64_t *sorted_experts,
                                 const int64_t *segment_offsets, const void *gate_weights,
                                 const void *gate_biases, const void *value_weights,
                                 const void *value_biases, const void *output_weights,
                                 const void *output_biases, void *output, int64_t pairs,
                                 int64_t input_width, int64_t hidden_width, int64_t expert_count,
                                 int dtype, void *workspace, size_t workspace_bytes,
                                 void *stream);

/* Combine sorted expert outputs into token rows: out[row] = sum of the row's
 * valid pair outputs / top_k, summed in sorted-pair order (deterministic, no
 * float atomics). out [tokens, width] in dtype.
 * Replaces moe/moe_kernels.cu:201-229,560-582 (combine_topk,
 * moe/__init__.py:315-360). Workspace: koemi_moe_combine_workspace(). */
KOEMI_API size_t koemi_moe_combine_workspace(int64_t tokens, int64_t pairs, int64_t top_k);
KOEMI_API int koemi_moe_combine_topk(const void *expert_outputs, const int64_t *sorted_rows,
                           const int64_t *segment_offsets, void *out, int64_t pairs,
                           int64_t width, int64_t tokens, int64_t top_k, int64_t expert_count,
                           int dtype, void *workspace, size_t workspace_bytes, void *stream);

/* Model-level fused combine: for each token row,
 *   u = context[row] + sum_slot scale_slot * expert_out[pair_positions[row*k+slot]]
 * over the row's valid pairs (pair_positions[p] < segment_offsets[E]), in
 * slot order, where scale_slot = weights[row*k+slot] (or 1/top_k when
 * weights is NULL); then out[row] = RMSNorm(u) * norm_weight where
 * valid[row], else context[row] (experts.py:136-142; router.py:70-73,96-97).
 * context/out fp32 [tokens, width]; expert_out in dtype. */
KOEMI_API int koemi_moe_combine_residual_rmsnorm(const float *context, const void *expert_out,
                                       const int64_t *pair_positions,
                                       const int64_t *segment_offsets, const float *weights,
                                       const uint8_t *valid, const float *norm_weight,
                                       float *out, int64_t tokens, int64_t width,
                                       int64_t top_k, int64_t expert_count, float eps,
                                       int dtype, void *stream);

/* The decode step's expert path with one permutation per step (the hash route
 * of every block is the same): koemi_moe_tile_prefix writes the grouped GEMMs'
 * tile map of segment_offsets (int32 [expert_count + 1], the 128-row tiles
 * before each expert) once, and koemi_moe_grouped_expert_mlp_mapped runs
 * koemi_moe_grouped_expert_mlp (tcgen05, bf16/f16 only) with that map, leaving
 * output rows past the valid pairs unwritten instead of zeroing them (the
 * combine never reads them). Workspace: koemi_moe_grouped_mlp_workspace.
 * Same reference lines as the grouped MLP (moe/__init__.py:179-312). */
KOEMI_API int koemi_moe_tile_prefix(const int64_t *segment_offsets, int64_t expert_count, int32_t *tile_prefix,
                                    void *stream);
KOEMI_API int koemi_moe_grouped_expert_mlp_mapped(const void *sorted_context, const int32_t *tile_prefix,
                                                  const int64_t *segment_offsets, const void *gate_weights,
                                                  const void *gate_biases, const void *value_weights,
                                                  const void *value_biases, const void *output_weights,
                                                  const void *output_biases, void *output, int64_t pairs,
                                                  int64_t input_width, int64_t hidden_width, int64_t expert_count,
                                                  int dtype, void *workspace, size_t workspace_bytes, void *stream);

/* The decode block's fusion RMSNorm (src/koemi/model/network.py:723-732)
 * fused with the row gather of its expert pairs: token row t of `fused` (fp32
 * [tokens, width]) is normalised, x * rsqrt(mean(x^2) + eps) * norm_weight,
 * into `context` (fp32; the arithmetic of koemi_core_rmsnorm_forward with fp32
 * in and out), and the normalised row is stored in rows_dtype (bf16/f16) at
 * rows_out[pair_positions[t * top_k + j]] for every pair below the valid count
 * (segment_offsets[expert_count]); other rows of rows_out are left as they were.
 * Width a multiple of 4 up to 2048. Replaces the norm plus a gather of the
 * sorted rows. */
KOEMI_API int koemi_moe_norm_gather(const float *fused, const float *norm_weight, float eps, float *context,
                                    const int64_t *pair_positions, const int64_t *segment_offsets,
                                    int64_t expert_count, void *rows_out, int rows_dtype, int64_t tokens,
                                    int64_t width, int64_t top_k, void *stream);

/* koemi_moe_combine_residual_rmsnorm for a chain of blocks: the combined,
 * normalised row x is stored as out_dtype, or, when next_norm_weight (fp32
 * [width]) is given, the next block's input RMSNorm(x) * next_norm_weight
 * (same eps) is stored instead, so x never goes to memory. Needs width % 4
 * == 0, width <= 2048, top_k <= 8, 16-byte aligned rows. No counterpart in
 * the reference (a fusion of two of its steps). */
KOEMI_API int koemi_moe_combine_residual_rmsnorm_next(const float *context, const void *expert_out,
                                            const int64_t *pair_positions,
                                            const int64_t *segment_offsets, const float *weights,
                                            const uint8_t *valid, const float *norm_weight,
                                            const float *next_norm_weight, void *out, int out_dtype,
                                            int64_t tokens, int64_t width, int64_t top_k,
                                            int64_t expert_count, float eps, int dtype, void *stream);

/* Sorted pair rows of a permutation already computed by koemi_moe_permute_topk:
 * out[i] = rows[sorted_rows[i]] converted from rows_dtype to out_dtype for
 * i < segment_offsets[expert_count], zero past it. Lets one permutation serve
 * several row sets (the hash route of a decode step is the same in every
 * block). Needs width % 4 == 0 and 16-byte aligned rows. */
KOEMI_API int koemi_moe_gather_rows(const void *rows, int rows_dtype, const int64_t *sorted_rows,
                          const int64_t *segment_offsets, int64_t expert_count, void *out, int out_dtype,
                          int64_t pairs, int64_t width, void *stream);

/* ---------------------------------------------------- expert parallelism */

/* Expert-parallel dispatch slab (no counterpart in the reference, which has
 * no expert parallelism). Rank g of `ranks` owns experts [g * local_experts,
 * (g + 1) * local_experts); the expert-major sorted pairs of
 * koemi_moe_permute_topk (sorted_rows [pairs, width], sorted_experts,
 * segment_offsets [ranks * local_experts + 1]) are therefore grouped by owner.
 * slab [ranks * capacity, width]: row g * capacity + j = sorted row
 * segment_offsets[g * local_experts] + j for j below owner g's count, with
 * slab_experts[g * capacity + j] = the owner-local expert id; padding rows get
 * slab_experts = -1 and are not written. capacity >= pairs (every pair may go
 * to one owner), so nothing is ever dropped. The slab is what an equal-split
 * all-to-all sends: block g to rank g. */
KOEMI_API int koemi_moe_ep_pack(const void *sorted_rows, const int64_t *sorted_experts,
                      const int64_t *segment_offsets, void *slab, int32_t *slab_experts,
                      int64_t pairs, int64_t width, int64_t ranks, int64_t local_experts,
                      int64_t capacity, int dtype, void *stream);

/* Inverse of koemi_moe_ep_pack for the returned expert outputs: sorted_out
 * [pairs, width] row i (i below segment_offsets[ranks * local_experts]) =
 * slab row g * capacity + (i - segment_offsets[g * local_experts]) with
 * g = sorted_experts[i] / local_experts; rows past the valid pairs are zero,
 * as koemi_moe_grouped_expert_mlp leaves them. */
KOEMI_API int koemi_moe_ep_unpack(const void *slab, const int64_t *sorted_experts,
                        const int64_t *segment_offsets, void *sorted_out, int64_t pairs,
                        int64_t width, int64_t ranks, int64_t local_experts, int64_t capacity,
                        int dtype, void *stream);

/* Fused expert-parallel exchange over peer memory (NVLink / NVSwitch), one
 * process per GPU, at most 8 ranks. Each rank allocates one exchange buffer of
 * koemi_peer_exchange_bytes() with koemi_peer_buffer_alloc, shares the
 * KOEMI_PEER_HANDLE_BYTES handle with the other ranks (any host channel) and
 * opens theirs with koemi_peer_buffer_open (CUDA IPC; no NVLink multicast
 * objects). `peers` is a device array [ranks] of every rank's buffer address
 * in this process (own buffer at [rank]); `own` is this rank's buffer.
 * One exchange, all ranks in the same order:
 *   koemi_ep_dispatch       sender: slab rows (the koemi_moe_ep_pack layout)
 *                           stored straight into the owners' buffers, then an
 *                           epoch flag per owner (release, system scope);
 *   koemi_ep_wait_dispatch  owner: waits for every sender's flag; the received
 *                           rows are then recv_rows [ranks * capacity, width]
 *                           with owner-local ids recv_ids (-1 padding) at the
 *                           buffer offsets of koemi_peer_exchange_offsets;
 *   koemi_ep_return         owner: the expert output of received row q
 *                           (local_out[local_positions[q]]) stored back into
 *                           its sender's buffer, then a flag per sender;
 *   koemi_ep_collect        sender: waits for every owner's flag and writes the
 *                           outputs in sorted pair order (zero past the valid
 *                           pairs), as koemi_moe_ep_unpack.
 * Every wait is bounded: a wait that runs out records KOEMI_ERR_TIMEOUT in the
 * device status word (koemi_device_status) and the kernel returns. No
 * counterpart in the reference, which has no expert parallelism. */
#define KOEMI_PEER_HANDLE_BYTES 64
KOEMI_API size_t koemi_peer_exchange_bytes(int64_t ranks, int64_t capacity, int64_t width, int dtype);
KOEMI_API int koemi_peer_exchange_offsets(int64_t ranks, int64_t capacity, int64_t width, int dtype,
                                size_t *ids_offset, size_t *rows_offset);
KOEMI_API int koemi_peer_buffer_alloc(size_t bytes, void **ptr, void *handle_out);
KOEMI_API int koemi_peer_buffer_open(const void *handle, void **ptr);
KOEMI_API int koemi_peer_buffer_close(void *ptr);
KOEMI_API int koemi_peer_buffer_free(void *ptr);
KOEMI_API int koemi_ep_dispatch(const void *sorted_rows, const int64_t *sorted_experts,
                      const int64_t *segment_offsets, const uint64_t *peers, void *own, int64_t pairs,
                      int64_t width, int64_t rank, int64_t ranks, int64_t local_experts,
                      int64_t capacity, int dtype, void *stream);

/* koemi_ep_dispatch fused with the row gather: slab row (g, j) is
 * context[sorted_tokens[i]] (context [tokens, width] in f32 or the exchange
 * dtype, converted to the exchange dtype on the way), so the sorted rows are
 * never written locally. 16-bit exchange rows, width a multiple of 8. */
KOEMI_API int koemi_ep_dispatch_gather(const void *context, int context_dtype, const int64_t *sorted_tokens,
                                       const int64_t *sorted_experts, const int64_t *segment_offsets,
                                       const uint64_t *peers, void *own, int64_t pairs, int64_t width, int64_t rank,
                                       int64_t ranks, int64_t local_experts, int64_t capacity, int dtype,
                                       void *stream);

/* koemi_ep_dispatch_gather fused with the RMSNorm that makes the rows: token
 * row t of `fused` (fp32 [tokens, width]) is normalised, x * rsqrt(mean(x^2)
 * + eps) * norm_weight, into `context` (fp32, the combine's residual; the
 * same arithmetic as koemi_core_rmsnorm_forward with fp32 in and out), and
 * each of its top_k pairs with a sorted index below the valid count (from
 * pair_positions, segment_offsets global [ranks * local_experts + 1]) is
 * stored, in the exchange dtype, into its owner's buffer; ids and epoch flags
 * as in koemi_ep_dispatch. 16-bit exchange rows, width a multiple of 4 up to
 * 2048. Replaces the block's fusion norm (src/koemi/model/network.py:723-732 in the
 * reference) plus the dispatch. */
KOEMI_API int koemi_ep_norm_dispatch(const float *fused, const float *norm_weight, float eps, float *context,
                                     const int64_t *pair_positions, const int64_t *sorted_experts,
                                     const int64_t *segment_offsets, int64_t tokens, int64_t top_k,
                                     const uint64_t *peers, void *own, int64_t width, int64_t rank, int64_t ranks,
                                     int64_t local_experts, int64_t capacity, int dtype, void *stream);

/* Owner side of an exchange in one launch: the bounded wait for every
 * sender's flag, then the stable sort of the received slots ([sender][j]) by
 * local expert and the gather of the live rows into expert-major order:
 * sorted_rows [ranks * capacity, width] (rows past the live count are left
 * as they were), segment_offsets [local_experts + 1], sorted_experts
 * [ranks * capacity] (local_experts for empty slots) and positions
 * [ranks * capacity] (sorted index of every slot). Optional (NULL: not
 * written): slots [ranks * capacity], the slot at every sorted index (the
 * inverse of positions), and tile_prefix [local_experts + 1] int32, the
 * number of 128-row tiles before each local expert (the tile map of
 * koemi_ep_expert_mlp_return). A wait that gives up records KOEMI_ERR_TIMEOUT
 * and yields empty segments. At most 4096 slots and 255 local experts.
 * Replaces koemi_ep_wait_dispatch plus a general permutation of the received
 * rows. */
KOEMI_API int koemi_ep_owner_sort(const uint64_t *peers, void *own, int64_t width, int64_t rank, int64_t ranks,
                                  int64_t local_experts, int64_t capacity, int dtype, void *sorted_rows,
                                  int64_t *segment_offsets, int64_t *sorted_experts, int64_t *positions,
                                  int64_t *slots, int32_t *tile_prefix, void *stream);

/* The owner's grouped gated expert MLP (koemi_moe_grouped_expert_mlp on
 * tcgen05 tensor cores, bf16/f16 only) over the rows of koemi_ep_owner_sort
 * (`rows` = ranks * capacity sorted rows, their segment_offsets, tile_prefix
 * and slots), whose output GEMM stores every live row's result straight into
 * its sender's exchange buffer (this owner's block of ret_rows, at the row's
 * slot) and then raises the return flag in every sender's buffer: it replaces
 * the grouped MLP, its output tensor and koemi_ep_return. Weights are this
 * rank's local experts in the grouped-MLP layout. workspace: at least
 * rows * hidden_width * 2 bytes (the gated hidden rows), 16-byte aligned. The
 * senders read the returned rows with koemi_ep_combine_residual_rmsnorm_next
 * (or koemi_ep_collect). Same reference lines as the grouped MLP. */
KOEMI_API int koemi_ep_expert_mlp_return(const void *sorted_rows, const int64_t *segment_offsets,
                                         const int32_t *tile_prefix, const int64_t *slots, const void *gate_weights,
                                         const void *gate_biases, const void *value_weights,
                                         const void *value_biases, const void *output_weights,
                                         const void *output_biases, int64_t rows, int64_t input_width,
                                         int64_t hidden_width, int64_t local_experts, int dtype, void *workspace,
                                         size_t workspace_bytes, const uint64_t *peers, void *own, int64_t rank,
                                         int64_t ranks, int64_t capacity, void *stream);

/* koemi_moe_combine_residual_rmsnorm_next for a sender of an exchange whose
 * owners returned their outputs with koemi_ep_expert_mlp_return: each CTA
 * waits (bounded) for every owner's return flag in `own`, then pair p's
 * expert row is read in place from the ret_rows block of the owner whose
 * segments hold p (segment_offsets are the global ones, expert_count = ranks
 * * local_experts). Replaces koemi_ep_collect, its sorted output tensor and
 * the combine's read of it. dtype: the exchange row type. */
KOEMI_API int koemi_ep_combine_residual_rmsnorm_next(const float *context, const int64_t *pair_positions,
                                                     const int64_t *segment_offsets, const float *weights,
                                                     const uint8_t *valid, const float *norm_weight,
                                                     const float *next_norm_weight, void *out, int out_dtype,
                                                     int64_t tokens, int64_t width, int64_t top_k,
                                                     int64_t expert_count, float eps, int dtype, const void *own,
                                                     int64_t ranks, int64_t local_experts, int64_t capacity,
                                                     void *stream);
KOEMI_API int koemi_ep_wait_dispatch(const void *own, int64_t ranks, void *stream);
KOEMI_API int koemi_ep_return(const void *local_out, const int64_t *local_positions, const uint64_t *peers,
                    void *own, int64_t width, int64_t rank, int64_t ranks, int64_t local_experts,
                    int64_t capacity, int dtype, void *stream);
KOEMI_API int koemi_ep_collect(const int64_t *sorted_experts, const int64_t *segment_offsets, void *sorted_out,
                     const uint64_t *peers, void *own, int64_t pairs, int64_t width, int64_t rank,
                     int64_t ranks, int64_t local_experts, int64_t capacity, int dtype, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* KOEMI_B200_H */
