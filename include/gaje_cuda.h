/*
 * gaje_cuda.h -- C ABI of the B200 decode engine for GAJE `.gaje.flat` v2 models.
 *
 * This is the drop-in boundary for the reference's decode path.  The reference
 * exposes that path only as Rust/PyO3 functions (its one C ABI, src/ffi.rs,
 * reaches redb `.gaje` sessions, not `.flat` files); each entry point below
 * names the reference function it replaces, by path:line inside the reference
 * project.  Conventions follow src/ffi.rs:13-90: opaque handles created by a
 * *_load call and released by the matching *_free, NULL on failure, every
 * pointer NULL-checked.  Because Result<_, String> has no C analogue, calls
 * return a status code (GAJE_OK == 0) and the message is available from
 * gaje_cuda_last_error() (thread-local).
 *
 * Threading: a gaje_model is not thread-safe (the reference methods take
 * &mut self).  Each model owns one CUDA stream, its KV cache and its scratch.
 *
 * Device errors become status codes: kernels never trap or assert.
 */
#ifndef GAJE_CUDA_H
#define GAJE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
enum gaje_status {
  GAJE_OK = 0,
  GAJE_ERR_INVALID = 1,     /* NULL pointer or argument out of range            */
  GAJE_ERR_IO = 2,          /* open/mmap failure, truncated file, bad magic,
                               malformed JSON (io::ErrorKind::InvalidData)       */
  GAJE_ERR_NOT_FOUND = 3,   /* tensor missing from the directory (NotFound)     */
  GAJE_ERR_SHAPE = 4,       /* tensor shapes/sizes inconsistent with the config */
  GAJE_ERR_UNSUPPORTED = 5, /* a format arm this engine does not implement      */
  GAJE_ERR_CUDA = 6,        /* CUDA runtime failure                             */
  GAJE_ERR_NAN = 7,         /* a NaN guard of src/nn/block/forward.rs fired      */
  GAJE_ERR_CONTEXT = 8,     /* KV cache full (max_ctx positions)                */
  GAJE_ERR_TIMEOUT = 9      /* a bounded device-side wait ran out               */
};

/* Thread-local message for the last failing call on this thread ("" if none). */
const char* gaje_cuda_last_error(void);

/* ------------------------------------------------------------- file format */
/* The fixed fields of FlatHeaderV2 (src/io/header/flat.rs:14-42). */
typedef struct gaje_flat_header {
  uint32_t version, flags, num_tensors;
  uint64_t meta_len, dir_len, weights_offset, weights_len;
  uint32_t group_size, quant_format;
  uint32_t arch_family, arch_n_embd, arch_n_head, arch_n_head_kv, arch_n_blocks,
      arch_qk_permute;
} gaje_flat_header;

/* The model configuration load_genomic derives (src/io/flat_reader.rs:124-142):
 * metadata JSON ModelConfig (src/io/config.rs:137-145) with the header's
 * ArchitectureDescriptor override (src/io/header/flat.rs:82-148). */
typedef struct gaje_flat_info {
  gaje_flat_header header;
  uint32_t n_embd, n_head, n_head_kv, n_blocks, head_dim, ffn_dim, vocab_size;
  float eps, rope_base;
  int rope_split;       /* 1 = "split" RoPE, 0 = "interleaved"              */
  int use_genomic_norm; /* ArchConfig.use_genomic_norm                        */
  int fused_qkv, fused_gate_up;
  int embd_bit_depth, lm_head_bit_depth, body_bit_depth;
  uint32_t n_entries;   /* tensors in the directory                         */
} gaje_flat_info;

/* Decodes the 4096-byte FlatHeaderV2 from memory (FlatHeaderV2::from_bytes,
 * src/io/header/flat.rs:47-60: only the magic is validated).  quant_format
 * 0/1/2 = LegacyCentroids/Q4_0/Q8_0 (flat.rs:62-70); a group_size of 0 means
 * the legacy 16 (flat.rs:73-79).  GAJE_ERR_IO on a short buffer or bad magic. */
int gaje_flat_header_decode(const uint8_t* bytes, size_t len, gaje_flat_header* out);

/* Parse-only open: header, metadata and directory, every tensor the loader
 * needs, offsets against the file size.  No device is touched.
 * Replaces GajeFlatFileReader::open + the validation part of load_genomic
 * (src/io/flat_reader.rs:33-69, 124-237). */
int gaje_flat_inspect(const char* path, gaje_flat_info* info);

/* The offline Q4_0 "Variant B" quantiser, 32 floats -> one 20-byte block
 * {f16 scale, f16 min, u8 qs[16]} (src/compute/quantize/python.rs:152-232).
 * n must be a multiple of 32; out holds n/32*20 bytes. */
int gaje_quantize_q4_0(const float* w, size_t n, uint8_t* out);
/* Q8_0, 32 floats -> {f16 scale, i8 qs[32]} (src/compute/quantize/python.rs:235-303). */
int gaje_quantize_q8_0(const float* w, size_t n, uint8_t* out);

/* `.gaje.flat` v2 writer with the layout of scripts/export_gaje_flat.py:184-483:
 * metadata JSON at 4096, directory JSON after it, 64-byte aligned blobs from a
 * 4 KiB aligned weights_offset, the packed 4096-byte header. */
typedef struct gaje_flat_writer gaje_flat_writer;
typedef struct gaje_flat_meta {
  const char* name;          /* config.name                                  */
  const char* tokenizer_id;  /* config.tokenizer_id                          */
  const char* tokenizer;     /* embedded tokenizer JSON string ("" if none)  */
  uint32_t arch_family;      /* 1 Llama, 2 SmolLM, 3 Qwen2, 4 Qwen2.5, 5 Gemma */
  uint32_t qk_permute;
  uint32_t n_embd, n_head, n_head_kv, n_blocks, vocab_size;
  float eps;
  double rope_base;
} gaje_flat_meta;
gaje_flat_writer* gaje_flat_writer_open(const char* path, const gaje_flat_meta* meta);
/* bit_depth 4 quantises to Q4_0, 8 to Q8_0, 32 stores raw f32.  bias may be NULL. */
int gaje_flat_writer_add_linear(gaje_flat_writer* w, const char* name, int bit_depth,
                                size_t out_features, size_t in_features,
                                const float* weights, const float* bias);
/* A norm vector (bit_depth 32, in_features 1), as the exporter writes them. */
int gaje_flat_writer_add_norm(gaje_flat_writer* w, const char* name, const float* v,
                              size_t n);
/* Writes header + metadata + directory + blobs; frees the writer. */
int gaje_flat_writer_close(gaje_flat_writer* w);

/* Seeded synthetic model: every matrix N(0, std), norms 1.0, optional QKV
 * bias N(0, std), tied embedding / lm_head written twice as the exporter does
 * (scripts/export_gaje_flat.py:338-341).  Body Q4_0, embeddings f32 or Q8_0. */
typedef struct gaje_synth_spec {
  uint32_t arch_family, n_embd, n_head, n_head_kv, n_blocks, ffn_dim, vocab_size;
  float eps;
  double rope_base;
  int qkv_bias;       /* 1: attn_qkv carries a bias (Qwen2 families)          */
  int embd_bit_depth; /* 32 (default) or 8                                    */
  float std;          /* 0 -> 0.02                                            */
  uint64_t seed;
} gaje_synth_spec;
int gaje_flat_write_synthetic(const char* path, const gaje_synth_spec* spec);

/* ------------------------------------------------------------------ model */
typedef struct gaje_model gaje_model;

typedef struct gaje_load_opts {
  int device;         /* CUDA device ordinal                                  */
  uint32_t max_ctx;   /* KV-cache capacity in positions; 0 -> 4096             */
  uint64_t seed;      /* sampling RNG seed for generate (temperature > 0)      */
  int use_graph;      /* kernel-per-phase engine: replay each step as a CUDA
                         graph (1, default) or launch kernel by kernel (0)    */
  int use_megakernel; /* 1 (default): one persistent cooperative kernel runs
                         whole decode steps -- the two-exchange-per-block
                         kernel when the shape fits it, else the five-exchange
                         one; 2: the five-exchange kernel only; 0: one kernel
                         per phase                                          */
  uint32_t max_streams; /* KV caches for gaje_cuda_forward_batch (0 = none)   */
  uint32_t max_prefill; /* rows of one gaje_cuda_prefill pass (0 = no prefill) */
} gaje_load_opts;
void gaje_load_opts_init(gaje_load_opts* opts);

/* load_genomic_auto (src/io/flat_reader.rs:240-251) for `.gaje.flat` files:
 * mmap, parse, repack on the device.  The returned model starts with the
 * reference's post-load state: K-WTA ratio 0.5 on the logits, 0.0 in the
 * blocks (src/io/flat_reader.rs:228-236, src/nn/block/init.rs:42).
 * NULL on error (gaje_cuda_last_error() says why). */
gaje_model* gaje_cuda_load(const char* flat_path, const gaje_load_opts* opts);
void gaje_cuda_free(gaje_model* model);

typedef struct gaje_model_info {
  uint32_t vocab_size, n_embd, n_head, n_head_kv, n_blocks, head_dim, ffn_dim;
  uint32_t max_ctx, cache_len;
  float eps, rope_base, k_wta_ratio;
  size_t device_bytes; /* weights + KV cache + scratch held on the device */
  uint32_t grid;        /* CTAs of the persistent kernel (one per SM) */
  uint32_t megakernel;  /* 2: the two-exchange persistent kernel, 1: the
                           five-exchange one, 0: one kernel per phase */
  uint32_t nranks, rank;           /* the vocab-sharded group (1, 0 when unsharded) */
  uint32_t vocab_row0, vocab_rows; /* lm_head rows this model holds */
} gaje_model_info;
int gaje_cuda_model_info(gaje_model* model, gaje_model_info* info);

/* GenomicLLM::forward_core (src/nn/llm/forward.rs:7-63): one decode step at
 * position = cache length.  logits_out (host, vocab_size floats) may be NULL;
 * argmax_out (host) may be NULL and receives the first index of the maximum
 * logit (the greedy choice of src/nn/llm/forward.rs:262-271). */
int gaje_cuda_forward(gaje_model* model, uint32_t token_id, int clear_cache,
                      float* logits_out, uint32_t* argmax_out);

/* generate_native_core (src/nn/llm/forward.rs:215-330): clears the cache,
 * prefills the prompt token by token, then greedy (temperature <= 1e-5) or
 * temperature sampling with repetition penalty, EOS stop and the 3x n-gram
 * repeat stop.  out holds max_new entries; *n_out receives the count.
 * Sampling draws from a seeded stream (the reference's thread_rng is not). */
int gaje_cuda_generate(gaje_model* model, const uint32_t* prompt, size_t n_prompt,
                       size_t max_new, float temperature, float repetition_penalty,
                       const uint32_t* eos_ids, size_t n_eos, uint32_t* out,
                       size_t* n_out);

/* clear_cache_core (src/nn/llm/forward.rs:174-178). */
int gaje_cuda_clear_cache(gaje_model* model);
/* set_k_wta_ratio (src/nn/llm/python.rs:53-59): model and every block. */
int gaje_cuda_set_k_wta_ratio(gaje_model* model, float ratio);
int gaje_cuda_set_seed(gaje_model* model, uint64_t seed);

/* Greedy decode kept on the device: n_steps forward steps, each fed the
 * previous step's argmax, the first fed first_token, with no host round trip
 * between steps (the loop of benchmarks/performance/bench_decode.py:182-192
 * with the argmax moved to the device).  tokens_out (host, n_steps entries,
 * nullable) receives the argmax of each step. */
int gaje_cuda_decode_greedy(gaje_model* model, uint32_t first_token, size_t n_steps,
                            uint32_t* tokens_out);

/* Batched decode (a few streams after long prompts, or hundreds of serving
 * streams): one forward_core step
 * (src/nn/llm/forward.rs:7-63) for each of B streams of the same model, each
 * with its own KV cache and position (its cache length).  stream_ids[B]
 * (distinct, < gaje_load_opts.max_streams) select the caches, tokens[B] are the
 * inputs; argmax_out[B] (host, nullable) receives each stream's greedy choice
 * (llm/forward.rs:262-271), logits_out (host, B x vocab_size, nullable) the
 * logits (with the logits K-WTA of :58-61 applied when its ratio is in (0,1)).
 * The weights of the step are read once for all B streams.  Block K-WTA and
 * use_genomic_norm are GAJE_ERR_UNSUPPORTED here; a full cache is
 * GAJE_ERR_CONTEXT.  Independent of the single-stream state (gaje_cuda_forward
 * and its cache). */
int gaje_cuda_forward_batch(gaje_model* model, const uint32_t* stream_ids, const uint32_t* tokens,
                            size_t B, uint32_t* argmax_out, float* logits_out);
/* The prompt part of generate_native_core (src/nn/llm/forward.rs:215-241)
 * for one batched stream: tokens[n] fed at positions len..len+n-1 (len = the
 * stream's cache length), as n consecutive forward_core steps would, but as
 * whole-prompt GEMMs on the tensor cores (gaje_load_opts.max_prefill rows at
 * a time) and a causal attention pass; argmax_out (host, nullable) and
 * logits_out (host, vocab_size, nullable) receive the last token's results
 * (logits K-WTA as gaje_cuda_forward_batch).  The stream's cache afterwards
 * holds the n new positions.  Needs max_prefill > 0; block K-WTA and
 * use_genomic_norm are GAJE_ERR_UNSUPPORTED; overflow is GAJE_ERR_CONTEXT. */
int gaje_cuda_prefill(gaje_model* model, uint32_t stream_id, const uint32_t* tokens, size_t n,
                      uint32_t* argmax_out, float* logits_out);
/* ------------------------------------------------- multi-GPU batched serving */
/* Request-parallel serving of many streams over several GPUs: one process
 * (or thread) per GPU, each holding the whole Q4 body and its own streams'
 * KV caches, and only a vocabulary slice of the f32 lm_head.  Each batched
 * step runs the body for the rank's own streams, all-gathers the residual
 * rows of every rank over NCCL, runs the output norm + lm_head slice for all
 * of them, all-gathers the per-row best (value, index) keys and keeps, per
 * local stream, the first maximum over the whole vocabulary: the same token
 * the single-GPU argmax (src/nn/llm/forward.rs:262-271) picks.  The
 * reference is single-process CPU code with no counterpart; the calls below
 * replace load_genomic_auto (src/io/flat_reader.rs:240-251) for one rank.
 *
 * Collective contract: every rank calls gaje_cuda_load_sharded together, and
 * then the same sequence of gaje_cuda_forward_batch / gaje_cuda_prefill calls
 * with the same B (each with its own streams and tokens).  A sharded model
 * returns argmax only (logits_out must be NULL: GAJE_ERR_UNSUPPORTED) and
 * refuses the single-stream calls (gaje_cuda_forward, _generate,
 * _decode_greedy, _profile_*, _trace_steps).  A collective that does not
 * finish within GAJE_NCCL_TIMEOUT_S seconds (environment, default 120) aborts
 * the communicator and the call returns GAJE_ERR_TIMEOUT; a failed NCCL call
 * returns GAJE_ERR_CUDA; either way the model must be reloaded.
 * NCCL is resolved at run time (dlopen of libnccl.so.2): a host process that
 * already loaded one shares it; GAJE_ERR_UNSUPPORTED when none is found. */
#define GAJE_NCCL_ID_BYTES 128
/* ncclGetUniqueId: one rank creates the id and the host hands it to the others. */
int gaje_cuda_nccl_unique_id(uint8_t* id_out /* GAJE_NCCL_ID_BYTES */);
/* gaje_cuda_load for rank `rank` of `nranks` (opts->device is this rank's GPU;
 * opts->max_streams must be > 0).  The lm_head rows held are those of
 * gaje_vocab_shard.  Collective: all ranks call it together.  NULL on error. */
gaje_model* gaje_cuda_load_sharded(const char* flat_path, const gaje_load_opts* opts, int nranks, int rank,
                                   const uint8_t* nccl_id /* GAJE_NCCL_ID_BYTES */);
/* Where a batched model's gaje_cuda_forward_batch steps spend their device
 * time, summed over the calls since the last reset (CUDA events on the model
 * stream, host round trips excluded).  Sharded model: ms_out[0] the body
 * (embedding rows through the last block), [1] the all-gather of the residual
 * rows, [2] output norm + this rank's lm_head rows + the per-row best keys,
 * [3] the all-gather of the keys + the merge.  One GPU: ms_out[0] the whole
 * step (body and head), [1..3] zero.  *steps_out (nullable) counts the calls;
 * reset != 0 zeroes both.  GAJE_ERR_INVALID without batched streams.  No
 * reference counterpart (the reference decodes one stream in one process). */
int gaje_cuda_batch_timings(gaje_model* model, float* ms_out /* [4] */, uint32_t* steps_out, int reset);
/* The vocabulary split: rank r holds lm_head rows [row0, row0 + rows) with
 * chunk = ceil(V / nranks), row0 = r * chunk. */
int gaje_vocab_shard(uint32_t vocab_size, int nranks, int rank, uint32_t* row0, uint32_t* rows);
/* The orderable argmax key the ranks exchange: larger value first, then the
 * lower index, so the largest key over all shards is the first maximum
 * (llm/forward.rs:262-271); NaN and -inf give 0 (never win); -0.0 == +0.0. */
uint64_t gaje_argmax_key(float value, uint32_t index);
uint32_t gaje_argmax_key_index(uint64_t key);

/* One batched step (the arguments of gaje_cuda_forward_batch, argmax and
 * logits not returned) launched kernel by kernel with CUDA events around each
 * kernel class: ms[GAJE_K_COUNT] receives the milliseconds spent in each
 * class (all blocks together), launches[GAJE_K_COUNT] the event brackets per
 * class (either may be NULL).  The streams advance as by a real step.  The
 * reference's counterpart is the GAJE_PROFILE_VERBOSE timing of
 * src/nn/llm/forward.rs:23-55. */
int gaje_cuda_profile_batch(gaje_model* model, const uint32_t* stream_ids, const uint32_t* tokens, size_t B,
                            float* ms, uint32_t* launches);

/* clear_cache_core for one batched stream. */
int gaje_cuda_clear_stream(gaje_model* model, uint32_t stream_id);
/* A batched stream's cache length. */
int gaje_cuda_stream_len(gaje_model* model, uint32_t stream_id, uint32_t* len);

/* The model's CUDA stream (a cudaStream_t), for callers that time it. */
void* gaje_cuda_stream(gaje_model* model);

/* Kernel classes of one decode step, for gaje_cuda_profile_steps. */
enum gaje_kernel_class {
  GAJE_K_QKV = 0, GAJE_K_ATTN = 1, GAJE_K_OPROJ = 2, GAJE_K_GATEUP = 3, GAJE_K_DOWN = 4,
  GAJE_K_LMHEAD = 5, GAJE_K_KWTA = 6, GAJE_K_COUNT = 7
};
/* Runs n_steps greedy steps like gaje_cuda_decode_greedy but launches each
 * kernel on its own, bracketed by CUDA events on the model stream, and writes
 * the mean milliseconds per step spent in each kernel class into
 * ms[GAJE_K_COUNT] and the launches per step into launches[GAJE_K_COUNT]
 * (either may be NULL).  The reference's counterpart is the
 * GAJE_PROFILE_VERBOSE timing of src/nn/llm/forward.rs:23-55. */
int gaje_cuda_profile_steps(gaje_model* model, uint32_t first_token, size_t n_steps,
                            float* ms, uint32_t* launches);

/* Phases of a megakernel step, for gaje_cuda_profile_phases. */
enum gaje_phase {
  GAJE_PH_QKV = 0, GAJE_PH_ATTN = 1, GAJE_PH_OPROJ = 2, GAJE_PH_GATEUP = 3, GAJE_PH_DOWN = 4,
  GAJE_PH_LMHEAD = 5, GAJE_PH_COUNT = 6
};
/* Runs n_steps greedy steps in one launch of the persistent decode kernel
 * with a %globaltimer stamp at the end of every phase on CTA 0, and writes the
 * mean microseconds per step spent in each phase (summed over the blocks) into
 * us[GAJE_PH_COUNT] and the whole-step mean into *step_us.  detail_us
 * (nullable, GAJE_PH_COUNT*5 floats) receives, per phase kind p, the mean
 * microseconds per step CTA 0 spent between consecutive trace points:
 *   [p*5+0] previous phase done -> phase entered
 *   [p*5+1] -> the input's publication flags seen
 *   [p*5+2] -> input staged in shared memory (attention: cached K/V landed)
 *   [p*5+3] -> rows done (attention: scores done)
 *   [p*5+4] -> outputs published
 * GAJE_ERR_UNSUPPORTED when the model runs on the kernel-per-phase engine.
 * The reference's counterpart is the GAJE_PROFILE_VERBOSE timing of
 * src/nn/llm/forward.rs:23-55. */
int gaje_cuda_profile_phases(gaje_model* model, uint32_t first_token, size_t n_steps,
                             float* us, float* step_us, float* detail_us);

/* The raw form of the above for every CTA: n_steps (<= 4096) greedy steps in
 * one launch; out[((cta*n_steps + step)*(5L+1) + 5l+p)*6 + k] is the
 * %globaltimer value (ns) of trace point k of phase p of block l (the lm_head
 * phase at 5L) on that CTA, 0 where the CTA had no work of that phase.  Points:
 * 0 entry, 1 input flags seen, 2 input staged (attention: cached K/V landed),
 * 3 rows done (attention: scores done), 4 outputs published, 5 first weight
 * slot ready.  out_len must be at least grid*n_steps*(5L+1)*6 (grid =
 * gaje_model_info.grid); *n_written receives the count.  No counterpart in the
 * reference: a diagnostic of the persistent kernel's critical path. */
int gaje_cuda_trace_steps(gaje_model* model, uint32_t first_token, size_t n_steps,
                          uint64_t* out, size_t out_len, size_t* n_written);

/* The same for the two-exchange persistent kernel (gaje_model_info.megakernel
 * == 2): out[((cta*n_steps + step)*(L+1) + l)*24 + k] is the SM cycle
 * count (clock64) of trace point k of block l on that CTA (0 where the CTA had
 * no such point).  Anchors map each CTA's cycles onto the global nanosecond
 * timer: out[(cta*n_steps*(L+1) + L)*24 + 22, 23] = (%globaltimer, clock64)
 * at the CTA's start, and the same row of the last step holds them at its
 * end in slots 20, 21.  Block points: 0 phase A entry, 1 input ready, 2 input staged,
 * 3 q (or k/v) rows done, 4 K/V rows landed, 5 attention done, 6 output
 * projection done, 7 split weights known, 8 phase A published, 9 phase B
 * input flags seen, 10 x_a formed, 11 staged, 12 first gate/up block done,
 * 13 down columns done, 14 phase B published, 15 split weight done, 16 the
 * split's attention starts, 17 scores done, 18 softmax done, 19 P*V done,
 * 20 next block's K/V rows requested (after 8), 21 the block input's flags
 * seen (blocks after the first).  l = L: 0 entry, 1 input ready, 2 staged, 3
 * lm_head rows done, 4 token published.  Slot 22 of (step 0, block 0) holds
 * the CTA's SM id (%smid) instead of a cycle count.  out_len must be at least
 * grid*n_steps*(L+1)*24.  No counterpart in the reference: a
 * diagnostic of the kernel's critical path. */
int gaje_cuda_trace_fused(gaje_model* model, uint32_t first_token, size_t n_steps,
                          uint64_t* out, size_t out_len, size_t* n_written);

/* The limit of every bounded device-side wait of this library's kernels on
 * `device` (mbarrier phases, exchange flags and words), in nanoseconds; 0
 * restores the default of 2 s.  A wait that runs out makes the call return
 * GAJE_ERR_TIMEOUT and leaves the CUDA context usable.  Applies to every model
 * on the device; call it while none of them is running a step.  No
 * counterpart in the reference (a CPU engine has no device waits). */
int gaje_cuda_set_wait_limit(int device, uint64_t ns);

/* Diagnostic of the failure path: in the model's next launch of the
 * two-exchange kernel, CTA `cta` (an attention CTA, 0 <= cta < n_head *
 * splits) raises no flag after the attention half of the first block, so
 * every other CTA's bounded wait for it runs out and the call returns
 * GAJE_ERR_TIMEOUT (after about two wait limits).  Applies to one launch;
 * the model's cache is then in an undefined state (clear it or reload).
 * GAJE_ERR_UNSUPPORTED when the model runs another engine.  No counterpart in
 * the reference. */
int gaje_cuda_debug_withhold_flag(gaje_model* model, int cta);

/* ---------------------------------------------------------------- op level */
/* Device-pointer entry points for the isolated kernel checks and sweeps.
 * `stream` is a cudaStream_t (NULL = legacy default stream). */

/* A Q4_0 matrix resident on the device in the engine's layout. */
typedef struct gaje_q4_matrix gaje_q4_matrix;
/* Uploads N rows of K/32 20-byte blocks (host memory, file layout) and an
 * optional bias[N] (host).  Replaces GenomicLinear::new's Q4_0 arm
 * (src/nn/linear/init.rs:29-35). */
gaje_q4_matrix* gaje_cuda_q4_0_upload(const uint8_t* blocks, size_t N, size_t K,
                                      const float* bias, int device);
void gaje_cuda_q4_0_release(gaje_q4_matrix* m);
/* y[m][n] = row_dot(n, x[m]) with the reference's |y|<1e-6 -> 0 flush and
 * +bias, for M input vectors x[M][K] (device) -> y[M][N] (device).
 * compute_single_row's Q4_0 arm (src/nn/linear/forward.rs:84-92, 113-115). */
int gaje_cuda_q4_0_gemv(const gaje_q4_matrix* m, const float* x, float* y, size_t M,
                        void* stream);
/* A Genomic4Bit matrix (the 16-centroid LUT format; GenomicLinear::new,
 * src/nn/linear/init.rs:29-38 and :109-124) uploaded for the op-level calls:
 * nibbles (host, N*K/2 bytes, element 2k in the HIGH nibble of byte k, as
 * genomize_4bit_core writes them) and centroids (host f32: 16 for the whole
 * matrix, K/32*16 per block column, or N*K/32*16 per row block).  The handle
 * works with gaje_cuda_q4_0_gemv (genomic_dot_product_4bit,
 * src/compute/kernels/genomic.rs:149-204, then the |t| < 1e-6 flush and the
 * bias; one launch per input vector), gaje_cuda_q4_0_dequant (w = c[code])
 * and gaje_cuda_q4_0_release.  NULL on error. */
gaje_q4_matrix* gaje_cuda_lut4_upload(const uint8_t* nibbles, const float* centroids, size_t n_centroids,
                                      size_t N, size_t K, const float* bias, int device);
/* Dequantised weights w[N][K] (device) with the AVX2 kernel's fused
 * fma(q, scale, min) (src/compute/kernels/genomic.rs:298). */
int gaje_cuda_q4_0_dequant(const gaje_q4_matrix* m, float* w, void* stream);

/* logits[n] = dot(x, W[n]) for an f32 W[N][K] (device), then the first index of
 * the maximum into *argmax (device u32).  logits may be NULL.
 * compute_single_row's F32 arm (src/nn/linear/forward.rs:20-32). */
int gaje_cuda_f32_gemv_argmax(const float* W, const float* x, size_t N, size_t K,
                              float* logits, uint32_t* argmax, void* stream);

/* rms_norm (src/compute/kernels/norm.rs:17-87): out = x * (1/sqrt(ss/n+eps)) * w. */
int gaje_cuda_rms_norm(const float* x, const float* w, float eps, size_t n, float* out,
                       void* stream);

/* Decode attention for one new position (src/nn/attention.rs:88-127): q[n_head*hd]
 * against ctx cached positions; k/v caches are [n_head_kv][cache_stride][hd]
 * (device).  out[n_head*hd].  q, k_cache, v_cache and out must be 16-byte
 * aligned (the cache rows are fetched with bulk copies) and head_dim a multiple
 * of 4; otherwise GAJE_ERR_INVALID / GAJE_ERR_UNSUPPORTED before any CUDA call.
 * A split whose copies do not land within the kernel's bounded wait (2 s)
 * leaves its KV-head group's outputs NaN; the next call starts clean. */
int gaje_cuda_attention_decode(const float* q, const float* k_cache, const float* v_cache,
                               size_t ctx, size_t cache_stride, size_t n_head,
                               size_t n_head_kv, size_t head_dim, float* out,
                               void* stream);

/* gaje_cuda_attention_decode without any device allocation, for callers that
 * must not allocate device memory on the call path: a host that budgets all of
 * its device memory at start-up, or one that cannot take the device-wide
 * synchronisation a cudaMalloc/cudaFree brings (gaje_cuda_attention_decode
 * allocates its per-device workspace on first use and re-allocates it, with a
 * device synchronise, when a larger geometry arrives).  No counterpart in the
 * reference, whose attention runs on the CPU.
 *
 * Same arguments, alignment rules, results and kernel as
 * gaje_cuda_attention_decode.  The split partials, the per-KV-head counters and
 * the per-KV-head timeout marks live in a 1 MiB buffer of static device memory
 * per device (held by every GPU that loads the library until the process
 * exits): the geometry must satisfy
 *   512 + n_head * 64 * (head_dim + 2) * 4 <= 1048576 bytes
 * (e.g. n_head 14 / head_dim 64, n_head 12 / head_dim 128); a larger one is
 * rejected with GAJE_ERR_UNSUPPORTED and a message giving both sizes.  The
 * counters and marks (the first 512 bytes) must be zero when a call starts:
 * they are zero when the library loads, and every call leaves them zero,
 * including one whose bounded wait ran out (that call's affected KV-head
 * group reads NaN in out; nothing else needs resetting).  The first call on a
 * device looks the buffer's address up with cudaGetSymbolAddress (with that
 * device current; it may load the module): make that first call before any
 * stream capture.  Every call repeats the lookup, which allocates nothing, so
 * the entry point stays usable after a cudaDeviceReset; the buffer then starts
 * from zero again.  Calls that overlap on the same device race on the one
 * buffer: serialise them (one stream, or events). */
int gaje_cuda_attention_decode_static(const float* q, const float* k_cache, const float* v_cache,
                                      size_t ctx, size_t cache_stride, size_t n_head,
                                      size_t n_head_kv, size_t head_dim, float* out,
                                      void* stream);

/* lateral_inhibition_kwta (src/compute/kernels/lut.rs:45-61) in place on
 * scores[n] (device): values below the k-th largest become -1e9. */
int gaje_cuda_kwta(float* scores, size_t n, size_t k, void* stream);

/* sample_top_p_core (src/compute/sampling.rs:14-55) on the device: logits[n]
 * (device) -> *token (device u32): p = exp((l - max) / temperature)
 * normalised, sorted by descending p (equal p in index order), the nucleus
 * cut after the first prefix whose sum exceeds top_p, then the first nucleus
 * token whose running sum reaches r * (the nucleus' sum).  r in [0, 1) is the
 * caller's uniform draw (the reference takes one from thread_rng, unseeded);
 * *kept (device u32, nullable) receives the nucleus size.  Sums are exact
 * (2^-40 fixed point), so the choice is deterministic; it can differ from the
 * reference's f32 running sums only where r or top_p is within their rounding
 * of a boundary.  One CTA, no scratch memory; n <= 2^23.  Asynchronous. */
int gaje_cuda_sample_top_p(const float* logits, size_t n, float temperature, float top_p, float r,
                           uint32_t* token, uint32_t* kept, void* stream);

/* quantize_q4_0_native (src/compute/quantize/python.rs:152-232) on the device:
 * w[n] (device f32, 16-byte aligned, n % 32 == 0) -> out (device, n/32 blocks
 * of 20 bytes, 4-byte aligned), the same bytes gaje_quantize_q4_0 writes on
 * the host.  Asynchronous on `stream`. */
int gaje_cuda_quantize_q4_0(const float* w, size_t n, uint8_t* out, void* stream);
/* The Q8_0 quantiser (python.rs, the 8-bit arm beside quantize_q4_0_native;
 * blocks.rs:37-50) on the device: n/32 blocks of 34 bytes (out 2-byte
 * aligned), the bytes of gaje_quantize_q8_0. */
int gaje_cuda_quantize_q8_0(const float* w, size_t n, uint8_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GAJE_CUDA_H */
