/*
 * detgpu.h -- C ABI of libdetgpu.so, the B200 (sm_100a) implementation of the
 * detllm token loop: teacher-forced Llama/Qwen2 forward -> logits -> integer
 * CDF for the range coder.
 *
 * This is the drop-in boundary.  Each entry point names the reference
 * interface it replaces (paths relative to the mii443/detllm repository).
 * The signatures use plain pointers and sizes only.  The caller owns every
 * host buffer; the library owns all device memory.
 *
 * Results are bit-identical to the reference CPU path: every f32 operation is
 * one explicitly rounded IEEE operation in the reference's order (no FMA
 * contraction, no fast-math), every reduction follows det-num's fixed 8-lane
 * tree, and transcendentals follow det-num's vendored fdlibm routines.
 *
 * Threading: a det_session is used by one host thread at a time.  Sessions on
 * different devices may run concurrently.  A det_model may back several
 * sessions on its device and may be shared by host threads: its model-level
 * codec calls (det_compress, det_decompress, det_encode_symbols) share one
 * session cached in the model, so concurrent calls on one model run one
 * after another.  det_model_free must not race with any call on the model.
 */
#ifndef DETGPU_H
#define DETGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t det_status;

/* ---- status codes ------------------------------------------------------- */
enum {
    DET_OK = 0,
    /* ModelError, crates/det-model/src/lib.rs:48-59 (declaration order) */
    DET_ERR_SHAPE = 1,
    DET_ERR_NONFINITE = 2,
    DET_ERR_UNSUPPORTED_ARCHITECTURE = 3,
    DET_ERR_UNSUPPORTED_HEAD_LENGTH = 4,
    DET_ERR_UNSUPPORTED_MODEL_FEATURE = 5,
    DET_ERR_UNSUPPORTED_ROPE_SCALING = 6,
    DET_ERR_MISSING_METADATA = 7,
    DET_ERR_GGUF = 8,
    DET_ERR_UNSUPPORTED_TENSOR_TYPE = 9,
    DET_ERR_THREAD = 10,
    /* CdfError, crates/det-coder/src/cdf.rs:10-17 */
    DET_ERR_CDF_EMPTY = 32,
    DET_ERR_CDF_MALFORMED = 33,
    DET_ERR_CDF_NONFINITE_LOGIT = 34,
    DET_ERR_CDF_SYMBOL_OUT_OF_RANGE = 35,
    DET_ERR_CDF_TOO_MANY_SYMBOLS = 36,
    DET_ERR_CDF_TOTAL_TOO_LARGE = 37,
    /* RangeError, crates/det-coder/src/range.rs:4-8 */
    DET_ERR_RANGE_INVALID_FREQUENCY = 40,
    DET_ERR_RANGE_UNEXPECTED_EOF = 41,
    /* FileError, crates/det-coder/src/file.rs:17-25 */
    DET_ERR_FILE_TOO_SHORT = 48,
    DET_ERR_FILE_BAD_MAGIC = 49,
    DET_ERR_FILE_UNSUPPORTED_VERSION = 50,
    DET_ERR_FILE_UNSUPPORTED_FLAGS = 51,
    DET_ERR_FILE_INVALID_CONTEXT = 52,
    DET_ERR_FILE_INVALID_OVERLAP = 53,
    /* compress/decompress driver, crates/det-cli/src/main.rs:433-855 */
    DET_ERR_TOKENIZER = 56,
    DET_ERR_WINDOW = 57,
    DET_ERR_MODEL_HASH_MISMATCH = 58,
    DET_ERR_NONCANONICAL = 59,
    DET_ERR_VOCAB_MISMATCH = 60,
    DET_ERR_DECODE = 61,
    DET_ERR_ALLOC = 62,
    DET_ERR_INVALID_ARGUMENT = 63,
    /* device side */
    DET_ERR_CUDA = 64,
    DET_ERR_NO_DEVICE = 65,
    DET_ERR_DEVICE_OOM = 66,
    DET_ERR_TIMEOUT = 67,
    DET_ERR_COLLECTIVE = 68,
    DET_ERR_SCRATCH_LIMIT = 69 /* request larger than a fixed scratch array */
};

/* RoPE pairing (det-model lib.rs:40-44) */
enum { DET_ROPE_ADJACENT = 0, DET_ROPE_SPLIT_HALF = 1 };

/* SymbolRange, crates/det-coder/src/cdf.rs:40-45 */
typedef struct {
    uint64_t cum;
    uint32_t freq;
    uint32_t reserved;
    uint64_t total;
} det_symbol_range;

/* LlamaConfig, crates/det-model/src/lib.rs:26-38, plus the tensor types */
typedef struct {
    uint32_t block_count, embedding_length, feed_forward_length;
    uint32_t head_count, head_count_kv, head_dim;
    uint32_t rope_dimension_count, rope_pairing;
    uint32_t context_length, vocab;
    float rms_epsilon, attention_scale, rope_freq_base;
    /* ggml types of token_embd, attn_q, attn_k, attn_v, attn_output,
     * ffn_gate, ffn_up, ffn_down, output (layer 0) */
    uint32_t weight_types[9];
    uint32_t has_qkv_bias, tied_output;
} det_config;

typedef struct det_model det_model;
typedef struct det_session det_session;

/* ---- library ------------------------------------------------------------- */
const char* det_status_string(det_status s);
/* number of visible CUDA devices (0 if none) */
det_status det_device_count(int* count);

/* ---- model: replaces F32Llama::from_gguf (det-model lib.rs:1035) --------- */
/* Parses the GGUF bytes (det-gguf lib.rs:156), validates the model exactly as
 * the reference does, uploads the weights to `device` in the library's
 * layout and keeps the GGUF's tokenizer (byte fallback, byte-level BPE or
 * SentencePiece, as det_tokenizer_kind reports) and the SHA-256 of the file
 * (det-cli main.rs:933-1008).  The bytes are not retained. */
det_status det_model_load(const uint8_t* gguf, size_t len, int device, det_model** out);
void det_model_free(det_model* model);
det_status det_model_info(const det_model* model, det_config* out);
/* SHA-256 of the GGUF bytes the model was loaded from */
det_status det_model_sha256(const det_model* model, uint8_t out[32]);

/* ---- tensor parallelism: the row partition of gemv_rows_parallel
 *      (det-model lib.rs:291-321) spread over devices ----------------------
 * Loads one replica of the model on each distinct device of
 * devices[0 .. n) (1 <= n <= 8; a device may repeat, which runs several
 * parts on one GPU) and returns a model whose sessions run one forward over
 * all n parts.  Part p computes a contiguous slice (64-row boundaries) of
 * the output rows of attn_output, ffn_gate, ffn_up, ffn_down and the
 * lm_head and, when head_count_kv is a multiple of n, its share of the KV
 * heads (their q/k/v rows, attention and KV cache); otherwise every part
 * runs the whole attention block.  Before each op that reads a whole row,
 * the parts exchange their slices (an all-gather: each part reads the
 * others' device memory over NVLink).  Every output row is the same
 * reduction as on one device, so logits, logits hashes and DTLZ streams are
 * identical to those of det_model_load's model.  The returned model and its
 * sessions take every other call unchanged; logits and CDF work stay on
 * devices[0].  det_model_free releases all replicas.
 * DET_ERR_COLLECTIVE: two of the devices cannot reach each other's memory. */
det_status det_model_load_tp(const uint8_t* gguf, size_t len, const int* devices, int n, det_model** out);

/* ---- session: replaces RopeTables::llama + KvCache::new + ForwardWorkspace
 *      (det-model lib.rs:813, 850, 963) ------------------------------------ */
/* n_ctx: positions per window (<= context_length); max_chunk: most
 * positions one det_forward call may process. */
det_status det_session_create(det_model* model, uint32_t n_ctx, uint32_t max_chunk, det_session** out);
void det_session_free(det_session* s);
/* fresh KV cache: KvCache::new for a window replay (det-cli main.rs:691-701) */
det_status det_session_reset(det_session* s);

/* ---- forward: replaces forward_one_with_workspace (det-model lib.rs:1249)
 * Teacher-forced: tokens[i] is processed at position pos0 + i, i < n.  The
 * n positions' logits stay on the device for det_symbol_ranges /
 * det_decoder_*; when logits_out is not NULL they are also copied to it as
 * n * vocab floats, row i = logits after tokens[i]. */
det_status det_forward(det_session* s, const uint32_t* tokens, uint32_t n, uint32_t pos0, float* logits_out);

/* ---- logits -> CDF: replaces logits_to_symbol_range_with_byte_escapes /
 *      logits_to_symbol_range_with_scratch (det-coder cdf.rs:108-136) -------
 * For i < n: out[i] = range of symbols[i] under the logits of row rows[i] of
 * the last det_forward (rows == NULL means row i). */
det_status det_symbol_ranges(det_session* s, const uint32_t* rows, const uint32_t* symbols, uint32_t n,
                             int byte_escapes, det_symbol_range* out);
/* ---- decoder side: replaces logits_to_decoder_distribution_with_* .total()
 *      and DecoderDistribution::symbol_range (det-coder cdf.rs:115-128,
 *      387-425), on the logits of row `row` of the last det_forward. */
det_status det_decoder_total(det_session* s, uint32_t row, int byte_escapes, uint64_t* total);
det_status det_decoder_lookup(det_session* s, uint32_t row, int byte_escapes, uint64_t value, uint32_t* symbol,
                              det_symbol_range* out);

/* ---- logits hash: replaces logits_hash_for_tokens_chunked (det-model
 *      lib.rs:1406); SHA-256 over the little-endian bits of every logit. --- */
det_status det_logits_hash(det_model* model, const uint32_t* tokens, size_t n, uint32_t chunk, uint8_t out[32]);

/* ---- compress / decompress: replaces det-cli compress / decompress
 *      (main.rs:433-511) including the windowed model state (:632-778) and
 *      the DTLZ container (det-coder file.rs).  n_ctx == 0 uses the model's
 *      context_length; overlap is n_ctx / 4.  *out is allocated by the
 *      library; release it with det_free. */
det_status det_compress(det_model* model, const uint8_t* input, size_t len, uint32_t n_ctx, uint8_t** out,
                        size_t* out_len);
det_status det_decompress(det_model* model, const uint8_t* dtlz, size_t len, uint8_t** out, size_t* out_len);
/* encode an explicit codec-symbol stream (symbols >= vocab are byte
 * escapes); returns the range-coder payload without header
 * (det-cli main.rs:523-552). */
det_status det_encode_symbols(det_model* model, const uint32_t* symbols, size_t n, uint32_t n_ctx, uint32_t overlap,
                              int byte_escapes, uint8_t** out, size_t* out_len);
void det_free(void* p);

/* ---- tokenizers: replace Tokenizer::from_gguf, tokenize_bytes,
 *      codec_symbols and decode_codec_symbol (det-token lib.rs:86-196,
 *      306-617).  Host only: they read the GGUF's tokenizer.ggml.* metadata
 *      and need no device.  kind: 0 byte fallback, 1 byte-level BPE
 *      (tokenizer.ggml.model "gpt2", or merges), 2 SentencePiece ("llama",
 *      "spm", "sentencepiece", or scores).  codec != 0 returns codec symbols
 *      (vocab + byte for a byte without a single-byte token); byte_escapes
 *      != 0 lets det_detokenize take those symbols.  *out is allocated by
 *      the library; release it with det_free.  Malformed tokenizer metadata
 *      and bytes or tokens the tokenizer cannot map return
 *      DET_ERR_TOKENIZER. */
det_status det_tokenizer_kind(const uint8_t* gguf, size_t len, int* kind);
det_status det_tokenize(const uint8_t* gguf, size_t len, const uint8_t* input, size_t n, int codec, uint32_t** out,
                        size_t* out_n);
det_status det_detokenize(const uint8_t* gguf, size_t len, const uint32_t* symbols, size_t n, int byte_escapes,
                          uint8_t** out, size_t* out_n);

/* ---- device numerics self-test: replaces `detllm selftest`'s canaries
 *      (det-cli main.rs:126-144) with a direct check of the device expf.
 * y[i] = det-num exp_f32(x[i]) (vendored_libm/expf.rs:33-106) computed on
 * `device`; n may be large (the exhaustive sweep uses 2^32 / k). */
det_status det_device_expf(int device, const float* x, float* y, size_t n);
/* Self-test of the tensor-parallel exchange's bounded wait (no counterpart
 * in the reference): on `device`, runs the exchange kernel waiting for a
 * peer counter that nothing sets.  The wait gives up after 2 s and the kernel
 * reports it through the error word, so the expected result is
 * DET_ERR_TIMEOUT, with the device still usable afterwards. */
det_status det_tp_exchange_timeout_selftest(int device);
/* Self-test of the bounded mbarrier waits of the bulk-copy pipelines (no
 * counterpart in the reference): on `device`, runs the tensor-core Q6_K
 * chunk GEMM on zero-filled records with one stage never copied.  Its waits
 * give up after 20 ms and the kernel reports it through the error word
 * (expected result DET_ERR_TIMEOUT), then the same launch with every stage
 * copied must finish without an error (else DET_ERR_CUDA). */
det_status det_q6k_pipeline_timeout_selftest(int device);
/* Measured latency of one dependent rounded f32 add on `device`, in SM
 * clock cycles (one warp, 8,192 adds between two clock reads, best of
 * three): the floor of every ordered chain, e.g. the K adds of a Q4_K row.
 * A benchmark hook with no counterpart in the reference. */
det_status det_add_latency_cycles(int device, double* cycles_per_add);

/* ---- timing hooks for benchmarks (device time of the last call) -------- */
typedef struct {
    double forward_ms;     /* device time inside det_forward kernels */
    double cdf_ms;         /* device time inside the CDF kernels */
    uint64_t launches;     /* library kernels launched */
    uint64_t h2d_bytes, d2h_bytes;
    uint64_t tokens;       /* positions forwarded */
    /* per-launch profile of the weight GEMV/GEMM kernels, filled only while
     * det_set_profiling(1): CUDA events around each launch on its stream */
    double gemm_ms;
    uint64_t gemm_launches;
    double gemm_bytes;     /* algorithmic bytes: weights + activations + outputs */
    double gemm_weight_bytes;
} det_stats;
det_status det_session_stats(det_session* s, det_stats* out, int reset);
/* sums of the stats of every session the model has run, including the ones
 * det_encode_symbols / det_compress / det_decompress / det_logits_hash make */
det_status det_model_stats(det_model* model, det_stats* out, int reset);
/* Weight-streaming rate of the one-token GEMVs in isolation: the weight
 * GEMV launches of one single-token forward (every matrix of every layer and
 * the lm_head, on the session's current activations) captured back to back
 * in one CUDA graph with programmatic dependent launch, replayed `reps`
 * times.  Returns the device time per pass and the algorithmic bytes per pass
 * (weights + quantised activations + outputs).  Overwrites the session's
 * logits: call det_forward again before det_symbol_ranges. */
det_status det_session_gemv_stream(det_session* s, uint32_t reps, double* ms_per_pass, double* bytes_per_pass);
/* Positions per forward chunk of det_encode_symbols / det_compress /
 * det_decompress's re-encode (16..1024; 0 restores the default, 1024 or
 * DETGPU_CHUNK).  The output bytes do not depend on it; it trades launch
 * count against parallel work per weight pass.  Process-wide; the previous
 * value goes to *previous when non-NULL.  A tuning hook with no counterpart
 * in the reference. */
det_status det_set_encode_chunk(uint32_t chunk, uint32_t* previous);
/* Chunk GEMM (more than 16 positions) for Q8_0 / Q4_0 weights: enable != 0
 * selects the tcgen05 tensor-core kernel, 0 the mma.sync kernel (the
 * default: faster at the shapes measured).  Both give identical bits.
 * Process-wide: models loaded while it is on get the kernel's weight copies
 * (as much device memory again as their Q8_0 / Q4_0 matrices), and their
 * forwards launched while it is on use them.  The previous setting goes to
 * *previous when non-NULL.  A tuning hook with no counterpart in the
 * reference. */
det_status det_set_q8_tensor_cores(int enable, int* previous);
/* per-launch device timing of every kernel (adds two event records per
 * launch and turns CUDA graphs off while enabled) */
det_status det_set_profiling(int enable);
/* The per-kernel profile gathered while profiling was enabled, summed over
 * the model's sessions, as a JSON object {"<kernel group>": [launches,
 * milliseconds], ...} written to out (cap bytes including the NUL). */
det_status det_model_profile(det_model* model, char* out, size_t cap, int reset);

/* ---- symbol ranges without allocation (no counterpart in the reference) --
 * For callers that cannot allocate device memory inside a call: engines that
 * fix their memory budget at start-up, runtimes whose allocator is not
 * cudaMalloc.  Same result as det_symbol_ranges with rows == NULL, but every
 * buffer is the caller's device memory: logits (n x vocab f32, row-major),
 * symbols (n u32) and out (n det_symbol_range).  Runs on the calling
 * thread's current device, on `stream` (a cudaStream_t; NULL = the legacy
 * default stream).  Every call ends by copying its error word to the host
 * and synchronising `stream`, on the error paths too, so it returns only
 * after its kernels have finished.
 * Working memory is one fixed array in device memory that every GPU loading
 * this library holds until exit: DET_NOALLOC_MAX_FLOATS floats of exp values
 * plus 2 * DET_NOALLOC_MAX_ROWS + 64 words, about 8 MiB.  Requests with
 * n > DET_NOALLOC_MAX_ROWS or
 * n * vocab > DET_NOALLOC_MAX_FLOATS return DET_ERR_SCRATCH_LIMIT.  The first
 * call on a device looks up the array's device address; make that first call
 * before any stream capture.  All calls on a device share the array: calls
 * whose work overlaps on the GPU race and must be ordered by the caller. */
#define DET_NOALLOC_MAX_ROWS 1024u
#define DET_NOALLOC_MAX_FLOATS (1u << 21)
det_status det_symbol_ranges_noalloc(const float* logits, uint32_t n, uint32_t vocab, const uint32_t* symbols,
                                     int byte_escapes, det_symbol_range* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif
