/*
 * qdec -- a B200 (sm_100a) decode engine for Qwen3.8-class hybrid models stored as K-quant GGUF files.
 *
 * C ABI.  Every function returns an int status: QDEC_OK (0) or a negative QDEC_E* code; qdec_last_error()
 * returns the message of the calling thread's last failure.  No C++ exception crosses this boundary.
 * Pointers named *_dev are device pointers; `stream` is a cudaStream_t (NULL = the legacy default stream).
 *
 * The reference engine (`aqueduct`, ManeeshJupalle/Qwen-3.8-in-Rust) is a Rust workspace with no FFI layer;
 * each entry point below names the crate API it replaces (paths relative to that project's root).
 */
#ifndef QDEC_H
#define QDEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QDEC_OK 0
#define QDEC_EINVAL (-1)   /* bad argument: shape, type, size (the reference's assert! panics) */
#define QDEC_ECUDA (-2)    /* a CUDA call failed */
#define QDEC_ENOMEM (-3)   /* device or host allocation failed */
#define QDEC_EIO (-4)      /* file I/O failed */
#define QDEC_EFORMAT (-5)  /* malformed GGUF or config contract violated (GgufError / ConfigError) */
#define QDEC_ESTATE (-6)   /* call out of order (e.g. spec_round before spec_prefill) */
#define QDEC_ETIMEOUT (-7) /* a device-side wait gave up; the kernel returned an error word */

/* ggml tensor types accepted by the kernels (GGUF type ids; crates/core/src/gguf.rs GgmlType) */
#define QDEC_TYPE_F32 0
#define QDEC_TYPE_Q4_0 2
#define QDEC_TYPE_Q8_0 8
#define QDEC_TYPE_Q4_K 12
#define QDEC_TYPE_Q5_K 13
#define QDEC_TYPE_Q6_K 14
/* Q6_K in the engine's split device layout: the tensor's 208-byte blocks [ql | qh | scales], then every block's
 * f16 d -- the same bytes as ggml's 210-byte blocks, 16-byte aligned for bulk copies (qdec_repack_q6k). */
#define QDEC_TYPE_Q6_K_SPLIT 114
/* The tile layout (qdec_repack_tiles): 8 rows x one super-block per tile block of 8 * (block bytes), arranged in
 * the order the GEMV threads read them; the same bytes as the ggml layout.  rows must be a multiple of 8. */
#define QDEC_TYPE_Q4_K_TILE 112
#define QDEC_TYPE_Q5_K_TILE 113
#define QDEC_TYPE_Q6_K_TILE 116
/* Q8_0 / Q4_0 in the tile layout: 8 rows x 8 blocks per tile block; rows % 8 == 0 and cols % 256 == 0. */
#define QDEC_TYPE_Q8_0_TILE 108
#define QDEC_TYPE_Q4_0_TILE 102

/* Library version string, e.g. "qdec 0.1.0 sm_100a". */
const char *qdec_version(void);
/* Message of the calling thread's last failed call ("" if none). */
const char *qdec_last_error(void);

/* ------------------------------------------------------------------------------------- kernel level */

/* Quantise `rows` rows of `n` f32 values (n % 256 == 0) into ggml block_q8_K rows
 * (per 256 values: f32 d, 256 x i8, 16 x i16 bsums; 292 bytes), bit-exact with the reference.
 * Replaces Q8KRow::quantize_into (crates/core/src/kernels/q8k.rs:51, :76-114). */
int qdec_quantize_q8k(const float *x_dev, int n, int rows, void *q8k_dev, void *stream);

/* Quantise into ggml block_q8_0 rows (per 32 values: f16 d, 32 x i8; 34 bytes), n % 32 == 0.
 * Replaces Q8Row::quantize_into (crates/core/src/kernels/q8.rs:65-103). */
int qdec_quantize_q8_0(const float *x_dev, int n, int rows, void *q8_dev, void *stream);

/* Size in bytes of one activation row of `cols` values in the form weights of `ggml_type` consume
 * (Q8_K for K-quants, Q8_0 for Q8_0/Q4_0, f32 for F32); 0 for an unsupported type.
 * Mirrors act_kind (crates/core/src/kernels/matvec.rs:147-160). */
size_t qdec_act_row_bytes(int ggml_type, int cols);

/* y[c * rows + r] = W[r] . act_c for c in [0, n_cols): the dequant-GEMV over pre-quantised activations.
 * `w_dev` is rows x cols in ggml row layout; `act_dev` holds n_cols activation rows of
 * qdec_act_row_bytes(type, cols) bytes each.  Every weight byte is read once per 4 columns.  Bit-exact with
 * matmul_fn / dot_q8k_t (crates/core/src/kernels/matvec.rs:377, :511-539; kdot.rs:314). */
int qdec_gemv(int ggml_type, const void *w_dev, int rows, int cols, const void *act_dev, int n_cols, float *y_dev,
              void *stream);

/* As qdec_gemv, from f32 activation rows (`x_dev`, n_cols x cols): each column is quantised into the form
 * the weight type consumes, then multiplied.  The quantised rows live in a device buffer the library owns
 * (one per device, grown on demand).  Replaces matvec_f32_in / matmul over ActVec
 * (crates/core/src/kernels/matvec.rs:541-545, :369-371). */
int qdec_matvec(int ggml_type, const void *w_dev, int rows, int cols, const float *x_dev, int n_cols, float *y_dev,
                void *stream);

/* The library's activation image (no counterpart in the reference; the same values as block_q8_K / block_q8_0
 * rows, rearranged for the GEMV): bytes of one row of `cols` values for weights of `ggml_type` (0 when the
 * type reads no image), quantising f32 rows into it, and the GEMV that reads it directly -- what qdec_gemv
 * does after rearranging block_q8_K / block_q8_0 columns, without that step.  K-quant types (ggml, split,
 * tile) read the Q8_K image, QDEC_TYPE_Q8_0_TILE / _Q4_0_TILE the Q8_0 image.  qdec_gemv_image wants the weights
 * and the image 16-byte aligned (QDEC_EINVAL otherwise). */
size_t qdec_image_row_bytes(int ggml_type, int cols);
/* Two K-quant tile matrices of the same shape against the same image columns in one launch (the MLP's gate and
 * up): y1[c * rows + r] = W1[r] . x_c, y2[c * rows + r] = W2[r] . x_c.  Replaces matvec2
 * (crates/core/src/kernels/matvec.rs:349) for the case x1 == x2 that mlp.rs:55 uses; the bits of each output are
 * those of qdec_gemv_image on that matrix alone. */
int qdec_gemv_image_pair(int ggml_type, const void *w1_dev, const void *w2_dev, int rows, int cols, const void *img_dev,
                         int n_cols, float *y1_dev, float *y2_dev, void *stream);
int qdec_quantize_image(int ggml_type, const float *x_dev, int n, int rows, void *img_dev, void *stream);
int qdec_gemv_image(int ggml_type, const void *w_dev, int rows, int cols, const void *img_dev, int n_cols, float *y_dev,
                    void *stream);

/* Tuning knob of the GEMV (process-wide; results do not depend on it -- it exists for tests and sweeps):
 *   impl 0 / 6: the kernel for ggml-layout Q4_K / Q5_K and split-layout Q6_K weights that reads the library's
 *     activation image (config 0 = automatic, 1..8 = lanes and rows per thread, depth, integer or FP32 scale
 *     multiply); impl 2: the kernel that reads block_q8_K activations in the reference layout instead;
 *   impl 7: the decode GEMV of K-quant tile matrices (config 0 = by shape, 1..8 = the streaming or windowed
 *     kernel with a fixed number of warps, tiles per warp, super-block phases and stages in flight);
 *   impl 8: the Q8_0 / Q4_0 tile kernel (config 0 = automatic, 1 = one warp per tile, 2 = the group range split
 *     over 4 warps, 3 = the same with two tiles per CTA);
 *   impl 9: the tensor-core prefill GEMM that K-quant tile matrices take for many columns (config = the smallest
 *     column count routed there, 16 by default, 0 = never; the 1..4 verify columns stay on the GEMV at any value
 *     >= 5);
 *   impl 10: the warp-MMA form of the Q4_K tile GEMV (integer lanes on mma.sync m16n8k32; config = the smallest
 *     column group routed there, 1..4, 4 by default, 0 = never).
 * No counterpart in the reference. */
int qdec_tune_gemv(int impl, int config);

/* Failure-handling self-test of one bounded device wait on the current device, in this process, without a peer
 * or a fault: `which` = 0 runs a tensor-parallel exchange step whose peer lines never arrive (they carry the
 * previous step's tag), 1 a decode GEMV whose first stage waits for bytes nothing sends (four runs: the streaming
 * and the windowed kernel, each in its dp4a and its warp-MMA form).  Each wait must give up after wait_ms
 * (1..10000), record its error word and let the kernel return with the context usable; the same work
 * is then run normally and must give the right result.  QDEC_OK when all of that held, QDEC_ECUDA (with the step
 * that misbehaved in qdec_last_error()) otherwise.  The engine's own waits give up the same way and surface as
 * QDEC_ETIMEOUT.  No counterpart in the reference (its CPU code has no device waits). */
int qdec_selftest_wait(int which, int wait_ms);

/* Repack rows x cols of ggml Q6_K (src) into the split layout (dst, the same number of bytes, a distinct
 * buffer) that qdec_gemv reads as QDEC_TYPE_Q6_K_SPLIT.  No counterpart in the reference (a device layout). */
int qdec_repack_q6k(const void *src_dev, int rows, int cols, void *dst_dev, void *stream);

/* Repack rows x cols of ggml Q4_K / Q5_K / Q6_K / Q8_0 / Q4_0 (src) into the tile layout (dst: the same number
 * of bytes, a distinct 16-byte aligned buffer) that qdec_gemv reads as QDEC_TYPE_*_TILE.
 * No counterpart in the reference (a device layout). */
int qdec_repack_tiles(int ggml_type, const void *src_dev, int rows, int cols, void *dst_dev, void *stream);

/* qdec_matvec for callers that cannot let a library allocate device memory: an application whose device memory
 * belongs to another allocator, or a decode loop that must stay allocation-free while it runs.  Same arguments,
 * same results as qdec_matvec, but the quantised columns live in a fixed array inside the library
 * (qdec_matvec_noalloc_max_bytes() bytes, held on every device that loads the library until exit); sizes that
 * do not fit are rejected with QDEC_EINVAL.  Bytes each column takes there, by the path the weights take:
 *   QDEC_TYPE_*_TILE K-quants, QDEC_TYPE_Q6_K_SPLIT and 16-byte aligned ggml Q4_K / Q5_K: cols/256 * 320
 *     (the library's Q8_K activation image);
 *   other K-quants (ggml Q6_K, unaligned Q4_K / Q5_K): cols/256 * 292 (block_q8_K rows);
 *   QDEC_TYPE_Q8_0_TILE / _Q4_0_TILE: cols/32 * 40 (the Q8_0 image);  ggml Q8_0 / Q4_0: cols/32 * 34 (block_q8_0);
 *   F32: none.
 * The first call on a device looks the array's address up and caches it, so make it before any stream capture;
 * cudaDeviceReset invalidates that cached address, so a process that resets a device must not call this entry
 * point on that device again.  All calls on a device share the array: calls that overlap on the GPU race.
 * This entry point has no counterpart in the reference, whose CPU matvec quantises into caller-owned rows. */
int qdec_matvec_noalloc(int ggml_type, const void *w_dev, int rows, int cols, const float *x_dev, int n_cols,
                        float *y_dev, void *stream);
size_t qdec_matvec_noalloc_max_bytes(void);
/* The scratch bytes qdec_matvec / qdec_matvec_noalloc need for n_cols columns of `cols` values against these
 * weights (the path depends on the type and on w_dev's alignment, as listed above); (size_t)-1 for a type or
 * width the kernels do not take.  A caller checks a noalloc call against qdec_matvec_noalloc_max_bytes() with
 * it.  No device work. */
size_t qdec_matvec_scratch_bytes(int ggml_type, const void *w_dev, int cols, int n_cols);

/* out[i * cols + e] = dequantised element e of row ids[i] of `w_dev` (ids on the device, n_ids of them):
 * the embedding gather.  Replaces Model::embed_token_into (crates/core/src/model.rs:364-368) and
 * dequantize_into (crates/core/src/quant.rs:229). */
int qdec_dequant_rows(int ggml_type, const void *w_dev, int rows, int cols, const int32_t *ids_dev, int n_ids,
                      float *out_dev, void *stream);


/* ------------------------------------------------------------------------------------- model level */

typedef struct qdec_model qdec_model;
typedef struct qdec_state qdec_state;

typedef struct qdec_opts {
    int device;   /* CUDA device ordinal */
    int max_pos;  /* positions the RoPE tables and KV caches of states cover (<= 0: 4096) */
} qdec_opts;

typedef struct qdec_model_info {
    uint32_t n_layer, hidden, ffn, vocab, n_head, n_head_kv, head_dim, dn_n_k_heads, dn_n_v_heads, dn_head_dim_k,
        dn_head_dim_v, n_full_attention, has_mtp;
    uint64_t weight_bytes;  /* bytes resident on the device */
    uint64_t decode_bytes;  /* weight bytes one plain token streams (layers + lm_head + norms + one embedding row) */
    uint64_t lm_head_bytes; /* output.weight */
    uint64_t mtp_bytes;     /* the MTP block's weights (blk.{n_layer}) */
    double load_secs;
} qdec_model_info;

/* Open a GGUF file and upload its tensors to the device: header, metadata and tensor index
 * (crates/core/src/gguf.rs:483), the config contract (crates/core/src/config.rs:146), the weights.
 * Replaces Model::load_with (crates/core/src/model.rs:184).  Malformed files give QDEC_EFORMAT with the
 * reference's GgufError / ConfigError message. */
int qdec_open(const char *gguf_path, const qdec_opts *opts, qdec_model **out);
/* 1 when the model's weights were read with O_DIRECT, bypassing the page cache (DirectFile,
 * crates/core/src/os.rs:311): opted into with the environment variable QDEC_LOAD_DIRECT=1, on one GPU, where the
 * file system allows O_DIRECT (not tmpfs); 0 when they were read through the page cache. */
int qdec_model_loaded_direct(const qdec_model *m);
/* Close a model.  With states of it still alive the model stays until the last of them is freed
 * (qdec_state_new on the closed model then fails with QDEC_ESTATE). */
int qdec_close(qdec_model *m);

/* Tensor parallelism over the GPUs of one node, one process per GPU (rank tp_rank of tp_world, 1..8).  Each
 * rank holds the output-row slices of every matrix (the reference's matvec row partition,
 * crates/core/src/kernels/matvec.rs:446-467, spread over GPUs instead of cores): the DeltaNet K heads and the V
 * heads tied to them, the attention q and kv heads, a 256-row range of the FFN, a range of the hidden-size
 * outputs and of the vocabulary.  Every row is computed whole, so the ids are those of one GPU; the sharded
 * activations are all-gathered between the ranks over peer memory.  A TP state must be connected
 * (qdec_tp_export on every rank, the handles gathered in rank order, qdec_tp_connect on every rank) before its
 * first prefill; all ranks then make the same calls with the same ids, and free their states only after every
 * rank's last call has returned.  QDEC_EFORMAT when the model's dimensions do not split over tp_world.
 * No counterpart in the reference (CPU-only, one process). */
int qdec_open_tp(const char *gguf_path, const qdec_opts *opts, int tp_rank, int tp_world, qdec_model **out);
/* The shard of rank tp_rank from the GGUF header alone (no device): out = {rank, world, kh_lo, nk, nv, qh_lo,
 * nq, kv_lo, nkv, ff_lo, ff_rows, h_lo, h_rows, v_lo, v_rows, 0} (first row / head and count of each range). */
int qdec_tp_plan(const char *gguf_path, int tp_rank, int tp_world, int32_t out[16]);
/* The same from the dimensions: dims = {hidden, ffn, vocab, n_head, n_head_kv, dn_n_k_heads, dn_n_v_heads,
 * has_deltanet_layers}. */
int qdec_tp_plan_dims(const uint32_t dims[8], int tp_rank, int tp_world, int32_t out[16]);
#define QDEC_TP_HANDLE_BYTES 80
int qdec_tp_export(const qdec_state *s, void *handle_out);
int qdec_tp_connect(qdec_state *s, const void *handles);
/* Exchange timing totals of a TP state (device clock, first thread of each exchange): {exchanges, ns writing
 * its slice to every rank, ns until the other ranks' lines had arrived, 0}. */
int qdec_tp_stats(const qdec_state *s, uint64_t out4[4]);
int qdec_model_get_info(const qdec_model *m, qdec_model_info *info);
/* Nonzero when `id` is a stop id: the GGUF EOS ids plus the architecture's (crates/core/src/arch.rs:79-90).
 * Replaces Model::is_stop (crates/core/src/model.rs:492). */
int qdec_is_stop(const qdec_model *m, uint32_t id);

/* A decode state for one sequence: spec_k > 0 adds the speculative buffers for k drafts per round
 * (Model::new_state / new_state_spec, crates/core/src/model.rs:334, spec.rs:184); max_pos bounds the
 * sequence (State::reserve, model.rs:123); max_rows bounds the rows of one forward (prefill chunk, >= k + 1).
 * A state is bound to one CUDA stream and is not thread-safe. */
int qdec_state_new(qdec_model *m, int spec_k, int max_pos, int max_rows, qdec_state **out);
int qdec_state_free(qdec_state *s);
int qdec_state_pos(const qdec_state *s);

/* Prefill `n` prompt ids; *first_out = argmax of the last row's logits (Model::prefill + logits_of +
 * argmax, crates/core/src/model.rs:443, :423, :505). */
int qdec_prefill(qdec_state *s, const uint32_t *ids, int n, uint32_t *first_out);
/* One token in, the greedy next token out; logits (vocab floats) copied to `logits_out` when non-null
 * (Model::forward_token, crates/core/src/model.rs:486). */
int qdec_step(qdec_state *s, uint32_t id, uint32_t *next_out, float *logits_out);
/* Multi-sequence batching on one GPU: one greedy step of each of `n` sequences in a single forward.  ids[i] is
 * fed to states[i] and next_out[i] receives its next token, exactly what qdec_step(states[i], ids[i], ..)
 * returns (each column of a batched matrix product is the single-row product bit for bit, the reference's
 * blocked matmul_t semantics, crates/core/src/kernels/matvec.rs:401-539).  Every weight matrix is read once
 * for the n rows; each row keeps its own state's conv window, DeltaNet state, KV cache and position.  The
 * states belong to one model on one GPU (no tensor parallelism), are greedy (no sampler), appear once each,
 * and states[0] was made with max_rows >= n (its row buffers carry the batch).  The reference decodes one
 * sequence at a time; this is an extension of qdec_step, with its error behaviour (QDEC_EINVAL on a bad
 * argument or a sequence at its max_pos, nothing advanced). */
int qdec_batch_step(qdec_state *const *states, int n, const uint32_t *ids, uint32_t *next_out);
/* Speculative prefill: prefill, x_T, the MTP over the prompt rows and the first k drafts; *x_out = x_T
 * (Model::spec_prefill, crates/core/src/spec.rs:229). */
int qdec_spec_prefill(qdec_state *s, const uint32_t *ids, int n, uint32_t *x_out);
/* One greedy speculative round from x_p: verify [x_p, d_1..d_k] in one batch, accept the longest matching
 * prefix plus the model's next token, roll back the DeltaNet states and KV length, re-feed the MTP and draft
 * the next round.  emitted_out receives *n_emitted (= m + 1 <= k + 1) ids; the last is the next x_p
 * (Model::spec_round, crates/core/src/spec.rs:326). */
int qdec_spec_round(qdec_state *s, uint32_t x_p, uint32_t *emitted_out, int *n_emitted);
/* Replace the drafts of the next round (k ids) -- the forced drafts of the identity tests
 * (Model::spec_set_drafts, crates/core/src/spec.rs:439); qdec_get_drafts reads the current ones. */
int qdec_set_drafts(qdec_state *s, const uint32_t *drafts, int k);
/* The state's sampler (SamplerConfig + Sampler::new / reseed, crates/core/src/sample.rs:58-170): temperature
 * <= 0 is greedy (the default); otherwise every emitted token is drawn as the reference draws it -- candidates
 * sorted by logit (ties: the lower id), the top_k of them (0: all), softmax at the temperature, top_p, min_p,
 * renormalised, one xoshiro256** uniform per draw -- and --spec k accepts drafts by the exact speculative rule
 * (accept_or_resample, sample.rs:279).  The RNG restarts from `seed`.  Set it before the first prefill of a
 * sequence.  QDEC_EINVAL on a tensor-parallel state (its logits are split over the ranks). */
int qdec_set_sampler(qdec_state *s, float temperature, int top_k, float top_p, float min_p, uint64_t seed);
int qdec_get_drafts(const qdec_state *s, uint32_t *drafts_out, int k);
/* The CUDA stream every kernel of this state runs on (to time it with events), and the number of kernels the
 * state has launched so far (for launch accounting); no counterpart in the reference (CPU-only). */
void *qdec_state_stream(const qdec_state *s);
uint64_t qdec_state_launches(const qdec_state *s);
/* Speculative counters: rounds, drafted, accepted, emitted (spec.rs:21-42 SpecStats). */
int qdec_spec_counters(const qdec_state *s, uint64_t out4[4]);

/* Parity hooks.  With capture on, every forward keeps the residual row after each layer; qdec_debug_hidden
 * copies row `row` after layer `layer` (layer == n_layer: the post-final-norm row) to host `out` (hidden floats).
 * qdec_debug_logits copies row `row` of the last forward's logits. */
int qdec_set_capture(qdec_state *s, int on);
int qdec_debug_hidden(qdec_state *s, int layer, int row, float *out);
int qdec_debug_logits(qdec_state *s, int row, float *out);
/* The carried state of layer `layer` after the last call, as the reference's State holds it (the deferred rows
 * of the last forward applied on a copy; the state itself is not changed) -- what the reference's
 * crates/core/tests/spec_identity.rs:5-9 compares after every round: what = 0 the DeltaNet recurrent state
 * f32 [n_v][dk][dv], 1 its conv window f32 [conv channels][conv_kernel - 1], 2 / 3 the K / V cache rows
 * [0, pos) f32 [pos][n_kv][head_dim] (a tensor-parallel rank: its own heads).  *n_floats: in, the capacity of
 * `out`; out, the floats written -- or, with out NULL, the floats needed (0 when the layer holds no such state). */
int qdec_debug_state(qdec_state *s, int layer, int what, float *out, size_t *n_floats);

/* Write a synthetic Qwen3.8-style GGUF (preset "tiny", "27b" or "27b-L<n>") seeded with `seed`, with
 * `threads` host threads (0 = all): the stand-in checkpoint of the benchmarks and parity tests. */
int qdec_synth_gguf(const char *path, const char *preset, uint64_t seed, int threads);

#ifdef __cplusplus
}
#endif
#endif /* QDEC_H */
