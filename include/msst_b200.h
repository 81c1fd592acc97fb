/*
 * msst_b200.h — C ABI of libmsst_b200, a B200-native (sm_100a) implementation of
 * the Roformer transformer stack of HuanLinOTO/CUDA-MSST-Infer
 * (MelBandRoformer and BS-Roformer: band split, axial time/band transformers,
 * mask estimators, mask merge).
 *
 * Conventions (all entry points):
 *   - plain pointers and sizes, no C++ types; device pointers unless named *_host
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream)
 *   - return MSST_OK (0) or an MSST_ERR_* code; msst_last_error() gives the
 *     message of the calling thread's last failure.  The reference throws
 *     std::runtime_error for the same conditions (src/tensor.h:28-34); its C++
 *     call sites get that behaviour back from a thin wrapper that throws on a
 *     non-zero status.
 *   - 16-bit operands are fp16 (MSST_F16) or bf16 (MSST_BF16); accumulation is
 *     fp32; the residual stream and all model inputs/outputs are fp32.
 *   - K (the reduction length) of every GEMM is a multiple of 64; hidden sizes
 *     of the Roformer (dim, heads*64, 4*dim) satisfy this, band inputs are padded.
 *   - head_dim is 64 on the Roformer path; msst_sdpa takes head_dim <= 64.
 *   - devices: a msst_model runs on the GPU it was loaded on; its device buffers
 *     must live on that GPU (or be managed memory), anything else is refused with
 *     MSST_ERR_INVALID before a kernel runs.  Op-level calls run on the GPU of
 *     their first operand.  Every call leaves the calling thread's current device
 *     as it found it.
 */
#ifndef MSST_B200_H
#define MSST_B200_H

#ifdef __cplusplus
extern "C" {
#endif

#define MSST_OK 0
#define MSST_ERR_INVALID 1     /* bad argument or unsupported shape            */
#define MSST_ERR_CUDA 2        /* CUDA runtime / cuFFT / driver error          */
#define MSST_ERR_IO 3          /* cannot read or parse a .csm file             */
#define MSST_ERR_UNSUPPORTED 4 /* model feature outside this implementation    */
#define MSST_ERR_DEVICE 5      /* a kernel's bounded wait gave up (see msst_device_error) */

#define MSST_F16 0
#define MSST_BF16 1
#define MSST_F32 2 /* output type of msst_layernorm only */

/* GEMM epilogues */
#define MSST_EPI_STORE16 0 /* out16 = act(x W^T + b)                               */
#define MSST_EPI_RESID32 1 /* out32 += x W^T + b   (residual add)                  */
#define MSST_EPI_STORE32 2 /* out32  = x W^T + b                                   */
#define MSST_EPI_GLU32 3   /* out32[j] = y[2j] * sigmoid(y[2j+1]), y = x W^T + b    */

#define MSST_ACT_NONE 0
#define MSST_ACT_GELU 1    /* erf form, src/ops_fused.cu:21-24 */
#define MSST_ACT_TANH 2
#define MSST_ACT_SIGMOID 3

#define MSST_AXIS_TIME 0
#define MSST_AXIS_BAND 1

/* msst_model_separate flags */
#define MSST_SEPARATE_FIX_TAIL_PADDING 1 /* pad the final short chunk from each channel's own
                                            samples instead of reproducing the reference's
                                            contiguous-source read (src/tensor.cu:377-405) */

typedef struct msst_model msst_model;

typedef struct msst_model_info {
  int model_type; /* 1 MelBandRoformer, 2 BSRoformer (app::ModelType order) */
  int dim, depth, heads, dim_head, num_bands, num_stems, channels;
  int n_fft, hop_length, sample_rate, chunk_size, num_overlap;
  int sum_band_dims; /* width of one mask row, sum over bands of 2*channels*freqs */
  int precision;     /* MSST_F16 or MSST_BF16 */
  /* config switches of the reference drivers (MBRConfig / BSRConfig::from_json) */
  int stft_normalized, skip_connection, match_input_audio_length;
  int bands_from_file; /* MelBandRoformer: 1 = __precomputed__ band tables of the .csm,
                          0 = computed at load (the reference's mel fallback) */
  float load_ms;       /* wall time of msst_model_load (read, convert, upload) */
} msst_model_info;

const char* msst_last_error(void);
/* Code recorded by a kernel whose bounded wait gave up (0 = none); clear != 0 resets it. */
unsigned msst_device_error(int clear);
int msst_version(void);
/* Number of kernels this library has launched (process-wide); reset != 0 returns and zeroes it. */
unsigned long long msst_kernel_launches(int reset);

/* Per-kernel timing of this library's launches, a measurement aid with no
 * counterpart in the reference.  msst_kernel_timing(1) discards earlier records
 * and starts recording: each launch is bracketed by two CUDA events on its stream
 * and tagged with its kernel name and its algorithmic FLOPs and DRAM bytes (the
 * operands read once and the results written once).  msst_kernel_timing(0) stops
 * recording.  msst_kernel_timing_report waits for the recorded launches, writes up
 * to `cap` per-name aggregates to `out` and the number of names to *count. */
typedef struct msst_kernel_stat {
  char name[40];
  unsigned long long launches;
  double total_ms;
  double flop;
  double bytes;
} msst_kernel_stat;
int msst_kernel_timing(int enable);
int msst_kernel_timing_report(msst_kernel_stat* out, int cap, int* count);

/* ---------------------------------------------------------------- op level -- */

/* RMSNorm of the reference, y = x * rsqrt(sum(x^2) + 1e-12) * gamma * scale
 * (replaces ops::rms_norm, src/ops_norm.cu:455-491).  x fp32 [rows, D]
 * (D % 128 == 0, D <= 1024) -> out16 [rows, D].  If wg != NULL also writes
 * gates[rows, heads] = sigmoid(y wg^T + bg) (the attention gate projection,
 * ops::linear_sigmoid at src/model_mel_band_roformer.cu:575). */
int msst_rmsnorm(const float* x, long long rows, int D, const float* gamma, float scale, int dtype, void* out16,
                 const float* wg, const float* bg, int heads, float* gates, void* stream);

/* out = epilogue(x W^T + b): x 16-bit [rows, K] (row stride ldx elements),
 * W 16-bit [N, K], bias fp32 [N] or NULL.  out is 16-bit for MSST_EPI_STORE16,
 * fp32 otherwise, row stride ldo.  Replaces ops::linear / linear_no_bias /
 * linear_gelu / linear_sigmoid (src/ops_linear.cu:150,349, src/ops_fused.cu:264,285)
 * and the residual Tensor::add_ (src/tensor.cu:1439). */
int msst_gemm(const void* x, long long rows, int K, long long ldx, const void* w, int N, const float* bias,
              int epilogue, int act, int dtype, void* out, long long ldo, void* stream);

/* QKV projection with the rotary embedding fused into the epilogue: qkv16
 * [rows, 3*heads*64] = x W^T with interleaved-pair rotation of the q and k
 * columns at position (row / pos_div) % pos_mod, tables cos/sin [pos_mod, 32]
 * (replaces linear_no_bias + split_qkv_heads + apply_rotary_emb,
 * src/model_mel_band_roformer.cu:540-559, src/ops_misc.cu:39-131). */
int msst_gemm_qkv_rope(const void* x, long long rows, int K, const void* w, int heads, const float* cos_tab,
                       const float* sin_tab, int pos_div, int pos_mod, int dtype, void* qkv16, void* stream);

/* Axial attention over a fused QKV buffer [B*T*F tokens, 3*heads*64] in
 * [B, T, F] token order: axis MSST_AXIS_TIME attends over t for every (b, f),
 * MSST_AXIS_BAND over f for every (b, t).  softmax(scale * q k^T) v, multiplied by
 * gates[token, head] when gates != NULL, heads merged: out16 [tokens, heads*64].
 * Replaces ops::scaled_dot_product_attention (src/ops_attention.cu:522-599) and
 * apply_gates_and_merge_heads (src/model_mel_band_roformer.cu:94-163). */
int msst_attention(const void* qkv16, int B, int T, int F, int heads, int axis, float scale, const float* gates,
                   int dtype, void* out16, void* stream);

/* ---- ops the reference shares with its conv model (HTDemucs' transformer,
 * src/model_htdemucs.cu:542-659); its linear and linear_gelu calls map to msst_gemm. */

/* LayerNorm over the last dimension, y = (x - mean) * rsqrt(var + eps) * gamma + beta
 * with the biased variance (replaces ops::layer_norm, src/ops_norm.cu:496-533;
 * the reference's default eps is 1e-5).  x fp32 [rows, D], D % 4 == 0 and
 * D <= 1024; out [rows, D] as out_dtype MSST_F32, MSST_F16 or MSST_BF16. */
int msst_layernorm(const float* x, long long rows, int D, const float* gamma, const float* beta, float eps,
                   int out_dtype, void* out, void* stream);

/* out = softmax(scale * q k^T) v per (batch, head), non-causal: q [B, H, Nq, d],
 * k and v [B, H, Nk, d], out [B, H, Nq, d], all 16-bit (dtype), d a multiple of 8
 * and <= 64; scale 0 selects 1/sqrt(d) (replaces ops::scaled_dot_product_attention,
 * src/ops_attention.cu:522-599, including its cross-attention form Nq != Nk). */
int msst_sdpa(const void* q, const void* k, const void* v, int B, int H, int Nq, int Nk, int head_dim, float scale,
              int dtype, void* out, void* stream);

/* One problem of msst_grouped_gemm: rows [a_row0, a_row0 + m) and columns
 * [a_col0, a_col0 + k) of x times rows [b_row0, b_row0 + n) (same k columns from
 * b_col0) of W, written to out rows out_row0.. and columns out_col0.. (for
 * MSST_EPI_GLU32 out_col0 counts output columns, n/2 per row); bias [n] or NULL. */
typedef struct msst_gemm_group {
  long long m, a_row0, out_row0;
  int n, k, a_col0, b_row0, b_col0, out_col0;
  const float* bias;
} msst_gemm_group;

/* Up to 64 independent GEMMs in one launch over one packed 16-bit x [x_rows, ldx]
 * and one packed 16-bit W [w_rows, ldw], all with the same epilogue (as
 * msst_gemm) into one output matrix out [out_rows, ldo].  Per group: k is a
 * multiple of 64 (pad K slices with zero columns); a_col0 and b_col0 are
 * multiples of 8 and out_col0 starts on 16 bytes (multiple of 8 for 16-bit, 4
 * for fp32 output).  The store / reduce epilogues write 32x32 blocks, so a
 * group's m (n) is a multiple of 32 unless its block ends at out_rows (ldo).
 * Replaces the reference's per-band GEMM loops of the band split and the mask
 * estimators (apply_band_split, apply_mask_estimator,
 * src/model_mel_band_roformer.cu:657-738, src/model_bs_roformer.cu:337-414),
 * which launch one cuBLAS GEMM per band. */
int msst_grouped_gemm(int num_groups, const msst_gemm_group* groups, const void* x, long long x_rows, long long ldx,
                      const void* w, long long w_rows, long long ldw, int epilogue, int act, int dtype, void* out,
                      long long out_rows, long long ldo, void* stream);

/* Device tables of a model's band gather and mask merge (read-only, owned by the
 * model; valid until msst_model_free).  Band b gathers nfreq[b] STFT bins
 * bin_list[bin_start[b] ..] into columns [kcol[b], kcol[b] + kpad[b]) of the
 * band-split input (2 * channels * nfreq[b] values, zero padding after), scaled
 * by gamma[gcol[b] ..].  Bin i of the mask merge sums the mask columns
 * contrib_col[contrib_off[i] .. contrib_off[i+1]) and divides by denom[i]. */
typedef struct msst_band_tables {
  int num_bands, nbins, channels, sum_kpad, sum_dims;
  const int* bin_start;
  const int* nfreq;
  const int* bin_list;
  const int* kcol;
  const int* kpad;
  const int* gcol;
  const float* gamma;
  const int* contrib_off;
  const int* contrib_col;
  const float* denom;
} msst_band_tables;
int msst_model_band_tables(const msst_model* m, msst_band_tables* tables);

/* Band gather + per-band RMSNorm (scale sqrt(band dims)) + 16-bit cast: spec is
 * the complex STFT in cuFFT R2C layout [B*C*T, nbins] (interleaved re/im fp32);
 * out16 [B*T, ldo] gets band b at columns [kcol[b], kcol[b] + kpad[b]) in the
 * reference's (bin, channel, re/im) order.  Replaces the per-band slice +
 * contiguous copy + rms_norm of apply_band_split and the mel-bin gather of
 * forward (src/model_mel_band_roformer.cu:657-690,808-829,
 * src/model_bs_roformer.cu:337-369,465-473). */
int msst_band_gather(const float* spec, int B, int T, const msst_band_tables* tables, int dtype, void* out16,
                     long long ldo, void* stream);

/* Mask merge: masks fp32 [S][B*T][sum_dims] (band-concatenated estimator output)
 * are averaged into bins (sum of the contributing bands / denom), multiplied
 * into the STFT spec [B*C*T, nbins] complex and written to out [(b*S + s)*C + c]
 * [T][nbins] complex (the iSTFT input), bin 0 zeroed when zero_dc != 0.
 * Replaces the scatter_add + average + complex multiply + zero-DC sequence of
 * forward (src/model_mel_band_roformer.cu:926-1015,
 * src/model_bs_roformer.cu:552-590). */
int msst_mask_apply(const float* spec, const float* masks, int B, int S, int T, const msst_band_tables* tables,
                    int zero_dc, float* out, void* stream);

/* ------------------------------------------------------------- model level -- */

/* Load a .csm model (format: src/weights.h:83-96) onto `device` with 16-bit
 * operands of type `precision` (replaces app::load_model,
 * src/inference_app.cpp:363-441, and the drivers' load(),
 * src/model_mel_band_roformer.cu:319-481, src/model_bs_roformer.cu:94-199). */
int msst_model_load(const char* path, int device, int precision, msst_model** out);
void msst_model_free(msst_model* m);
int msst_model_get_info(const msst_model* m, msst_model_info* info);

/* Whole forward pass on device buffers: audio [batch, channels, length] fp32 ->
 * out [batch, num_stems, channels, (length/hop)*hop] fp32 (the stem axis is
 * absent from the reference's shape when num_stems == 1; the memory layout is
 * the same).  Replaces MelBandRoformer::forward / BSRoformer::forward
 * (src/model_mel_band_roformer.cu:744, src/model_bs_roformer.cu:420). */
int msst_model_forward(msst_model* m, const float* audio, int batch, int channels, long long length, float* out,
                       void* stream);

/* Forward steps up to the mask estimators: fp32 masks
 * [batch, num_stems, T, sum_band_dims], T = length/hop + 1. */
int msst_model_masks(msst_model* m, const float* audio, int batch, int channels, long long length, float* masks,
                     void* stream);

/* One axial transformer (all its layers, plus the MelBandRoformer's final norm)
 * applied in place to the residual stream x fp32 [batch, T, num_bands, dim]
 * (replaces apply_transformer, src/model_mel_band_roformer.cu:628-651,
 * src/model_bs_roformer.cu:310-331, with the permutes of forward() folded away). */
int msst_model_transformer(msst_model* m, int depth_index, int axis, float* x, int batch, int T, void* stream);

/* Block level, in place on the residual stream x fp32 [batch, T, num_bands, dim]:
 * layer `layer` of the transformer (depth_index, axis).  The attention block is
 * RMSNorm + gate projection, QKV + RoPE, attention with gates and head merge, out
 * projection and residual add (replaces apply_attention + the residual add of
 * apply_transformer, src/model_mel_band_roformer.cu:519-591,628-651,
 * src/model_bs_roformer.cu:236-284,310-331); the feed-forward block is RMSNorm,
 * Linear + GELU, Linear and residual add (apply_feedforward,
 * src/model_mel_band_roformer.cu:597-622, src/model_bs_roformer.cu:290-304).
 * Neither applies the MelBandRoformer's per-transformer final norm
 * (msst_model_transformer does). */
int msst_roformer_attn_block(msst_model* m, int depth_index, int axis, int layer, float* x, int batch, int T,
                             void* stream);
int msst_roformer_ffn_block(msst_model* m, int depth_index, int axis, int layer, float* x, int batch, int T,
                            void* stream);

/* msst_model_transformer for callers that cannot allocate device memory while
 * they run: real-time audio hosts, whose processing callback has a hard deadline
 * that a cudaMalloc / cudaFree (which can block and synchronise the device)
 * would break, and applications that own every device allocation themselves.
 * There is no counterpart in the reference.  All intermediates live in one
 * fixed 48 MiB device array inside the library (held on every GPU that loads
 * it, until exit); nothing is allocated.  A call over batch*T*num_bands tokens
 * needs about dim*2 + heads*4 + 2*max(3*heads*64, 4*dim) + heads*128 bytes per
 * token (about 10,000 tokens at dim 384) and larger calls fail with
 * MSST_ERR_INVALID.  Calls on one device share the array: calls that overlap on
 * the GPU race.  The first call on a device looks up the array's device address,
 * and under CUDA's lazy module loading it is also when the driver loads the
 * library's module and backs the array with device memory: make one warm-up
 * call per device at start-up, off the real-time thread and before any stream
 * capture.  Later calls allocate nothing and do not synchronise the stream. */
int msst_model_transformer_noalloc(msst_model* m, int depth_index, int axis, float* x, int batch, int T,
                                   void* stream);

/* Chunked overlap-add separation of one track (replaces app::run_inference /
 * process_chunked, src/inference_app.cpp:100-324,443-497).  track [channels,
 * length] -> out [num_stems, channels, length].  overlap: (0,1) = overlap
 * ratio, >= 1 = num_overlap, 0 = model default.  chunk_batch <= 0 uses the
 * reference default (2).  *_host variants take host memory (copies included). */
int msst_model_separate(msst_model* m, const float* track, int channels, long long length, float overlap,
                        int chunk_batch, int flags, float* out, void* stream);
int msst_model_separate_host(msst_model* m, const float* track_host, int channels, long long length, float overlap,
                             int chunk_batch, int flags, float* out_host);

/* Sharded separation of one track across GPUs (the reference is single-GPU;
 * these split msst_model_separate at its independent unit, the chunk).
 * msst_model_forward_chunks runs chunks [first_chunk, first_chunk + count) of the
 * track's chunk plan: track [channels, length] (device) -> out [count,
 * num_stems*channels, chunk_size] (device).  msst_model_stitch overlap-adds the
 * outputs of all chunks of the plan, chunks [num_chunks, num_stems*channels,
 * chunk_size], into out [num_stems, channels, length], in chunk order, so the
 * result equals msst_model_separate's. */
int msst_model_forward_chunks(msst_model* m, const float* track, int channels, long long length, float overlap,
                              int first_chunk, int count, int chunk_batch, int flags, float* out, void* stream);
int msst_model_stitch(msst_model* m, const float* chunks, int channels, long long length, float overlap, float* out,
                      void* stream);

/* Round-robin sharding (chunk i on rank i % world, the reference's chunk list of
 * src/inference_app.cpp:131-137 dealt out): msst_model_forward_chunks over chunks
 * first_chunk, first_chunk + chunk_stride, ... (count of them). */
int msst_model_forward_chunks_strided(msst_model* m, const float* track, int channels, long long length,
                                      float overlap, int first_chunk, int chunk_stride, int count, int chunk_batch,
                                      int flags, float* out, void* stream);

/* The overlap-add of msst_model_stitch (src/inference_app.cpp:252-306,
 * src/ops_fused.cu:138-188) for output samples [begin, end) only, written into
 * out [num_stems, channels, length] (other samples untouched).  Chunk k's output
 * [num_stems*channels, chunk_size] is read from slot (k % slot_ranks) * slot_cap +
 * k / slot_ranks of `chunks` (slot_ranks = 1, slot_cap = num_chunks: chunk order;
 * slot_ranks = world: each rank's round-robin shard after the previous rank's).
 * Each sample is summed over its chunks in chunk order, so stitching a track in
 * ranges gives the same result as one msst_model_stitch. */
int msst_model_stitch_range(msst_model* m, const float* chunks, int slot_ranks, int slot_cap, int channels,
                            long long length, float overlap, long long begin, long long end, float* out,
                            void* stream);

/* Sample ranges of chunk `chunk_index` of a track's plan.  in_ranges[4] receives
 * two ranges [begin, end) of the track its gather reads: its own reflect-padded
 * window, and (only for a short final chunk with the reference's padding, i.e.
 * without MSST_SEPARATE_FIX_TAIL_PADDING) the first samples of the track that
 * padding reads, else an empty range.  [*out_begin, *out_end) is the output its
 * overlap-add touches: output samples before chunk k's out_begin are final once
 * chunks 0..k-1 are stitched. */
int msst_model_chunk_span(const msst_model* m, long long length, float overlap, int chunk_index, int flags,
                          long long* in_ranges, long long* out_begin, long long* out_end);

/* Chunk plan of msst_model_separate for a track length (src/inference_app.cpp:119-138). */
int msst_model_chunk_plan(const msst_model* m, long long length, float overlap, int* chunk_size, int* step,
                          long long* border, long long* padded_length, int* num_chunks);

#ifdef __cplusplus
}
#endif

#endif /* MSST_B200_H */
