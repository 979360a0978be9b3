/* s3t — SAM 3 ViT vision trunk on NVIDIA B200 (sm_100a): the C ABI.
 *
 * Drop-in for the reference's vision-trunk entry point
 *   sam3::VisionTrunk::run(image_nchw, shape_nchw)
 *   (include/sam3/vision_trunk.h:15-26, src/vision_trunk.cpp:297-488),
 * reading the same GGUF tensors (names resolved through the converter's
 * <file>.tensor_map.json sidecar like src/gguf_model.cpp:28-47,190-204) in the
 * same F32 / F16 / Q8_0 formats.
 *
 * Conventions follow the reference's C API (include/sam3/c_api.h,
 * src/c_api.cpp:19-23): functions return 0 on success and -1 on failure with
 * a thread-local message from s3t_last_error(); nothing throws across the ABI;
 * buffers passed in are borrowed, never freed.  One context is bound to one
 * GPU and is not safe for concurrent calls (like the reference's
 * VisionTrunk::run, which shares the backend's work buffer).
 */
#ifndef S3T_H
#define S3T_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type codes of the weight formats (ggml/include/ggml.h GGML_TYPE_*). */
enum { S3T_TYPE_F32 = 0, S3T_TYPE_F16 = 1, S3T_TYPE_Q8_0 = 8 };

/* s3t_trunk_run flags: where the image and output buffers live. */
enum {
    S3T_IMAGES_ON_DEVICE = 1, /* images_nchw is a device pointer on the context's GPU */
    S3T_OUTPUT_ON_DEVICE = 2, /* out_nchw is a device pointer on the context's GPU */
};

typedef struct s3t_ctx s3t_ctx;

/* Create a context on CUDA device `device`.  Replaces GgufModel::load's
 * backend selection (src/gguf_model.cpp:107-120) for the trunk.  NULL on error. */
s3t_ctx *s3t_create(int device);
void s3t_destroy(s3t_ctx *ctx);
const char *s3t_last_error(void);

/* Stage one trunk tensor (host bytes, ggml layout: ne[0] fastest).  `name`
 * is the original (unhashed) tensor name, e.g.
 * "backbone.vision_backbone.trunk.blocks.3.attn.qkv.weight".  Replaces the
 * per-tensor ggml_backend_tensor_set of src/gguf_model.cpp:150-153. */
int s3t_set_weight(s3t_ctx *ctx, const char *name, int ggml_type, const int64_t ne[4], const void *host_bytes,
                   size_t nbytes);

/* Read every trunk tensor of a GGUF file (GgufModel::load,
 * src/gguf_model.cpp:83-168).  tensor_map_path may be NULL, meaning
 * "<gguf_path>.tensor_map.json" if that file exists. */
int s3t_load_gguf(s3t_ctx *ctx, const char *gguf_path, const char *tensor_map_path);

/* Check a GGUF file as s3t_load_gguf reads it, without a GPU: header,
 * metadata, tensor records and every trunk tensor's type and byte range
 * against the file's length.  Outputs (may be NULL): the number of trunk
 * tensors and of transformer blocks found.  A truncated or corrupt file
 * returns -1 with a message, like GgufModel::load returning false
 * (src/gguf_model.cpp:83-94). */
int s3t_gguf_inspect(const char *gguf_path, const char *tensor_map_path, int *n_trunk_tensors, int *n_layers);

/* Validate shapes/types of the staged tensors, upload them and convert them
 * to the GEMM operand format (Q8_0 / F32 -> fp16 on the device, patch-embed
 * repacked).  Must be called once before the first run. */
int s3t_finalize_weights(s3t_ctx *ctx);

/* Number of transformer blocks found in the weights (32 for SAM 3). */
int s3t_num_layers(const s3t_ctx *ctx);

/* The trunk: images [batch][3][1008][1008] fp32 -> out [batch][1024][72][72]
 * fp32, both NCHW (VisionTrunk::run, src/vision_trunk.cpp:297-488, with the
 * batch of 1 generalised to `batch` independent images).  stream is a
 * cudaStream_t or NULL for the context's own stream.  With host buffers the
 * call returns after the output is in host memory; with both buffers on the
 * device it returns after enqueueing (check with s3t_sync). */
int s3t_trunk_run(s3t_ctx *ctx, const float *images_nchw, int batch, float *out_nchw, int flags, void *stream);

/* Same, stopping after the first n_layers blocks (0 = patch embed + pos +
 * ln_pre only).  Mirrors the per-stage dumps of the reference's
 * tools/export_vision_trunk_reference.py (.stem/.ln_pre/.layer_NN). */
int s3t_trunk_run_layers(s3t_ctx *ctx, const float *images_nchw, int batch, int n_layers, float *out_nchw, int flags,
                         void *stream);

/* One block of the trunk from a given residual: x_dev [batch*5184][1024]
 * fp32 token-major (token y*72 + x of each image, the input of block
 * `layer`) -> out_dev, the same layout, the block's output residual
 * (norm1, attention with its window partition, proj + residual, norm2, MLP
 * + residual: one iteration of the layer loop of src/vision_trunk.cpp:377-459).
 * Per-block parity entry, the counterpart of the per-layer dumps of the
 * reference's tools/export_vision_trunk_reference.py.  Device pointers on
 * the context's GPU; synchronous (returns after the block ran). */
int s3t_trunk_run_block(s3t_ctx *ctx, int layer, const float *x_dev, int batch, float *out_dev, void *stream);

/* The trunk from decoded 8-bit RGB: rgb [batch][height][width][3] uint8
 * (row-major HWC, what stbi_load returns; all images of a call share one
 * size) is resized and normalized on the device exactly as the reference's
 * load_image_rgb (src/pipeline.cpp:45-83; tools/sam3_vision_trunk.cpp:33-66
 * bilinear_resize_rgb) and then run through the trunk, replacing the host
 * preprocessing loop and the 12 MB fp32 image per request.  flags as for
 * s3t_trunk_run: S3T_IMAGES_ON_DEVICE means rgb is a device pointer.
 * 1 <= width, height <= 32768.  Image decoding (stbi_load) stays with the
 * caller. */
int s3t_trunk_run_rgb8(s3t_ctx *ctx, const uint8_t *rgb, int width, int height, int batch, float *out_nchw,
                       int flags, void *stream);

/* No counterpart in the reference: one eager (not graph-replayed) trunk run on
 * device buffers with a CUDA event after every launch, for measurement.
 * Returns per kernel class the summed device milliseconds and the launch
 * count, in this order: 0 stem (im2col + patch GEMM + ln_pre/norm1),
 * 1 QKV GEMM, 2 windowed attention, 3 global attention, 4 proj GEMM,
 * 5 LayerNorm, 6 fc1 GEMM, 7 fc2 GEMM.  kind_ms and kind_launches hold 8
 * entries each.  Synchronous. */
int s3t_trunk_profile(s3t_ctx *ctx, const float *images_dev, int batch, float *out_dev, void *stream,
                      double *kind_ms, int *kind_launches);

/* Wait for the context's queued work and report any device-side error. */
int s3t_sync(s3t_ctx *ctx, void *stream);

/* --- the vision neck's first operation, on the trunk's device output -------
 * The reference hands the trunk's output to sam3::VisionNeck::run as a host
 * vector (src/pipeline.cpp:159-163, src/vision_neck.cpp:203-206), a full D2H
 * and H2D in between.  These take the trunk's NCHW output where
 * s3t_trunk_run (S3T_OUTPUT_ON_DEVICE) left it and run the first operation of
 * one neck level (src/vision_neck.cpp:262-345) with the neck weights the same
 * GGUF file holds (backbone.vision_backbone.convs.*):
 *   level 0: 2x2 stride-2 transposed conv dconv_2x2_0 + bias, then GELU
 *            (the input of the second transposed conv) -> [B][512][144][144]
 *   level 1: 2x2 stride-2 transposed conv dconv_2x2 + bias -> [B][512][144][144]
 *   level 2: 1x1 conv conv_1x1 + bias                      -> [B][256][72][72]
 *   level 3: 2x2 max pool, then 1x1 conv conv_1x1 + bias   -> [B][256][36][36]
 * (channel counts as the file gives them; s3t_neck_first_shape reports them).
 * trunk_dev [batch][1024][72][72] and out_dev are fp32 device memory of the
 * context's GPU; enqueued on `stream` (NULL: the context's own stream).  The
 * operands are fp16 with fp32 accumulation and the result passes through
 * fp16.  The transposed conv multiplies the values in the order the
 * reference's graph reads them (its ggml_permute(x, 2, 0, 1, 3) on [W, H, C],
 * :96-105).  Uses the context's workspace: not concurrently with a trunk run
 * on the same context. */
int s3t_neck_first(s3t_ctx *ctx, int level, const float *trunk_dev, int batch, float *out_dev, void *stream);

/* Shape [1][C][H][W] of s3t_neck_first's output for one image, or -1 if the
 * file holds no weights for that level. */
int s3t_neck_first_shape(const s3t_ctx *ctx, int level, int64_t shape[4]);

/* --- several GPUs of one node -------------------------------------------
 * No counterpart in the reference, which runs the trunk on one backend device
 * (src/gguf_model.cpp:107-120).  The trunk is per image, so a batch is split
 * into contiguous shards of ceil(batch / n_devices) images, one per GPU; each
 * GPU holds its own copy of the weights and is driven by its own host thread.
 * The only exchange is moving images in and feature maps out (peer copies,
 * no collective inside the trunk).  A handle is not safe for concurrent calls. */
typedef struct s3t_multi s3t_multi;

/* Load the trunk of gguf_path onto every listed device (distinct device
 * indices; devices[0] is the "first GPU" below).  NULL on error. */
s3t_multi *s3t_multi_create(const int *devices, int n_devices, const char *gguf_path, const char *tensor_map_path);
void s3t_multi_destroy(s3t_multi *m);
int s3t_multi_num_devices(const s3t_multi *m);

/* images [batch][3][1008][1008] -> out [batch][1024][72][72] fp32 NCHW.  Host
 * buffers (flags 0): every GPU copies its own slices in and out; returns when
 * the output is in host memory.  With S3T_IMAGES_ON_DEVICE /
 * S3T_OUTPUT_ON_DEVICE the buffers are memory of devices[0]: the other GPUs
 * peer-copy their images in and their features out (the gather to the first
 * GPU), chunk by chunk so the copies overlap their compute.  `stream` is a
 * stream of devices[0] (NULL: its context's own stream); with device buffers
 * the call returns after enqueueing, and that stream waits for every GPU's
 * work (check with s3t_multi_sync). */
int s3t_multi_run(s3t_multi *m, const float *images_nchw, int batch, float *out_nchw, int flags, void *stream);

/* Wait for every GPU's queued work of the handle and report device errors. */
int s3t_multi_sync(s3t_multi *m, void *stream);

/* --- op-level entry points (parity tests, microbenchmarks) --------------- */

/* Dequantize GGUF weight bytes on the device to fp32: F16 and Q8_0
 * (dequantize_row_q8_0, ggml/src/ggml-quants.c:436-450).  Device pointers. */
int s3t_dequantize(int ggml_type, const void *src_dev, int64_t n, float *dst_dev, void *stream);

/* The fp16 GEMM operand that s3t_finalize_weights makes of a linear weight,
 * with the same conversion: Q8_0 -> fp16(q * d) (the exact product of
 * dequantize_row_q8_0, ggml/src/ggml-quants.c:436-450, rounded to nearest
 * even fp16), F32 -> fp16 (round to nearest even), F16 -> unchanged.
 * Device pointers; dst16 holds n fp16 values. */
int s3t_weight_operand(int ggml_type, const void *src_dev, int64_t n, void *dst16_dev, void *stream);

/* y16[M][N] = fp16(act(x16[M][K] * w16[N][K]^T + bias)) — the trunk's GEMM
 * (ggml_mul_mat + bias, src/vision_trunk.cpp:50-62).  act: 0 none, 1 GELU-erf.
 * q8: apply the Q8_0 activation rounding to the output.  Device pointers. */
int s3t_gemm_f16(int device, const void *x16, const void *w16, const float *bias, int M, int N, int K, int act,
                 int q8, void *y16, void *stream);

/* Flash attention on grouped, already-rotated q/k/v [groups*16][L][64]
 * (fp16 or bf16), output token-major [images*5184][1024] in natural token
 * order (windowed: 9 groups per image).  Device pointers. */
int s3t_attention(int device, const void *q, const void *k, const void *v, int groups, int L, int windowed, int bf16,
                  void *out, void *stream);

/* Multi-head attention of the encoder fusion, 8 heads of 32 (model width
 * 256): replaces mha() of src/encoder_fusion.cpp:63-88, the
 * ggml_flash_attn_ext call with prec F32 and scale 1/sqrt(32) that the
 * encoder's self attention (:266, no mask) and image-to-prompt cross
 * attention (:299, prompt mask) run.  `batch` independent sequences (the
 * reference runs one image per call; batch 1 is that call): q_dev
 * [batch][q_len][256], k_dev/v_dev [batch][kv_len][256] token-major fp16
 * (flags & S3T_MHA_BF16: bf16), head h in columns [32h, 32h+32).
 * key_mask_dev: null, or [batch][kv_len] fp32 added to every query row's
 * scaled scores; a key whose entry is -inf takes no part (the reference
 * builds its prompt mask as 0 / -inf rows of this vector, :120-133), and a
 * row whose keys are all masked gives 0, as ggml's CPU kernel does.  out_dev
 * [batch][q_len][256] fp32, or the operand type with S3T_MHA_OUT_F16.
 * Device pointers, 16-byte aligned, on `device`, enqueued on `stream`.
 * Returns 0, or -1 with s3t_last_error(). */
#define S3T_MHA_BF16 1
#define S3T_MHA_OUT_F16 2
/* With S3T_MHA_BIAS, key_mask_dev is a full additive bias [batch][8][q_len]
 * [kv_len] fp32 (one row per sequence, head and query): the decoder's image
 * cross attention with its box relative-position bias (mha() of
 * src/decoder.cpp:95-127 over image_bias_t, :401-418, :457-465).  The
 * decoder's other two attentions are the plain call: self attention over its
 * 201 queries (:430, no mask) and the text cross attention with the prompt
 * mask row (:443).  The decoder computes softmax explicitly (ggml_soft_max_ext):
 * the result is the same, except that a row with every key at -inf is NaN
 * there and 0 here.
 * Scratch: when the query tiles cannot fill the GPU and there are 16 or more
 * blocks of 64 keys (the decoder's 201 queries against 5184 image tokens),
 * each tile's keys are split into ranges computed in parallel and merged;
 * the call then allocates a stream-ordered scratch buffer of about
 * batch * ceil(q_len / 128) * 128 * 8 heads * splits * 34 floats
 * (cudaMallocAsync on `stream`, freed with cudaFreeAsync on the same stream;
 * 5.3 MB for that decoder call, split 19 ways).  Every other call allocates
 * nothing. */
#define S3T_MHA_BIAS 4
int s3t_mha_d32(int device, const void *q_dev, const void *k_dev, const void *v_dev, int batch, int q_len,
                int kv_len, const float *key_mask_dev, void *out_dev, int flags, void *stream);

/* The preprocessing of s3t_trunk_run_rgb8 alone: rgb_dev [batch][height]
 * [width][3] uint8 -> out_dev [batch][3][1008][1008] fp32, bit-exact with
 * the reference's bilinear_resize_rgb (tools/sam3_vision_trunk.cpp:33-66).
 * Device pointers on `device`, enqueued on `stream`. */
int s3t_preprocess_rgb8(int device, const uint8_t *rgb_dev, int width, int height, int batch, float *out_dev,
                        void *stream);

/* Axial RoPE in place on grouped q or k (layout as above). */
int s3t_rope(int device, void *x, int groups, int L, int windowed, int bf16, void *stream);

/* LayerNorm over 1024 columns (eps 1e-5), fp32 in -> fp16 out (q8: Q8_0
 * activation rounding of the output).  Device pointers. */
int s3t_layernorm(int device, const float *x, int rows, const float *gamma, const float *beta, void *y16, int q8,
                  void *stream);

/* No counterpart in the reference: failure-detection self-test.  One device
 * thread waits, for limit_ms (1..2000), on an mbarrier that nothing arrives
 * at; the bounded wait gives up, records a timeout in the device status word
 * and the kernel returns.  Returns 0 when the wait gave up as designed; the
 * next s3t_device_status(device) then reports (and clears) the timeout, and
 * the device stays usable. */
int s3t_selftest_wait_timeout(int device, int limit_ms);

/* Synchronize `device` and report (then clear) the device status word that
 * the op-level entry points write when a bounded in-kernel wait times out. */
int s3t_device_status(int device);

/* Allocation-free stem (no counterpart in the reference): patch embedding +
 * tiled position embedding + ln_pre for one image, the same values as
 * s3t_trunk_run_layers(ctx, ..., n_layers = 0, ...) but token-major:
 * images_dev [batch][3][1008][1008] fp32 -> out_tokens_dev [batch*5184][1024]
 * fp32, both device pointers on the context's GPU and 16-byte aligned,
 * enqueued on `stream` (NULL = the context's own stream, as for every other
 * entry point that takes a context).  For callers that cannot call
 * cudaMalloc (plugins whose host application owns all device memory, loops
 * with a fixed memory budget): it allocates nothing; its one scratch buffer
 * is a static device array inside the library sized for batch <= 1
 * (6,635,520 bytes, held by every GPU that loads the library until exit).
 * Larger batches are rejected with an error.  The first call on a device
 * looks up that array's device address; make that first call before any
 * stream capture.  Calls whose work overlaps on the same GPU race on the
 * shared array. */
int s3t_stem_noalloc(s3t_ctx *ctx, const float *images_dev, int batch, float *out_tokens_dev, void *stream);

#ifdef __cplusplus
}
#endif
#endif
