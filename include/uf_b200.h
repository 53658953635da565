/*
 * uf_b200.h -- C ABI of the B200 (sm_100a) INT16 engine for the DCVC-UF HT-L
 * per-frame hot path.
 *
 * Arithmetic contract: "uf-int16-q9-w13-acc64-rna-sat-v1" (reference
 * include/uf/int16_ops.hpp:10-13): features Q9, weights Q13, exact int64 dot
 * products, rna(sum / 8192) with ties away from zero, + int16 Q9 bias, int16
 * saturation.  Results are bit-identical to the reference's CPU path.
 *
 * Conventions
 *   - Operator entry points take DEVICE pointers to dense NCHW tensors (the
 *     reference's torch::Tensor layout), plain sizes, and a cudaStream_t passed
 *     as void* (NULL = the legacy default stream).  They are asynchronous on
 *     that stream; the caller owns every input and output buffer.
 *   - Return value: 0 on success, a negative UFB_E* code on failure; the
 *     message is available from ufb_last_error() (thread-local).  Argument
 *     checks mirror the reference's TORCH_CHECKs and are done before any launch.
 *   - Kernel pipeline timeouts (a bounded wait that gave up) are recorded in a
 *     per-device status word read by ufb_device_status().
 */
#ifndef UF_B200_H
#define UF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UFB_OK 0
#define UFB_EINVAL -1   /* invalid argument (reference: std::invalid_argument / TORCH_CHECK) */
#define UFB_ERANGE -2   /* size exceeds an indexing or exactness bound (std::overflow_error) */
#define UFB_ECUDA -3    /* CUDA runtime error */
#define UFB_ESTREAM -4  /* corrupt or truncated entropy-coded stream (std::runtime_error) */
#define UFB_ESTATE -5   /* call not valid in the current codec state (std::runtime_error) */

/* Library version (major * 10000 + minor * 100 + patch). */
int ufb_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* ufb_last_error(void);

/* Synchronise `device` and return then clear its kernel status word:
 * 0 when no kernel reported a pipeline timeout since the last call, else the
 * first recorded code (1..4 = TMA producer / MMA / epilogue / drain wait). */
int ufb_device_status(int device);

/* ---------------------------------------------------------------------------
 * Operators.  Each replaces one function of the reference's CUDA extension,
 * include/uf/cuda_ops.hpp:10-23 (definitions src/cuda/conv.cu:114-135 and
 * src/cuda/elementwise.cu:49-98), with the same argument meaning and checks;
 * the output is caller-allocated instead of returned.
 * ------------------------------------------------------------------------- */

/* uf_conv (include/uf/cuda_ops.hpp:10-12): exact INT16 convolution.
 * x [n, ci, h, w], weight [co, ci/groups, kh, kw], bias [co] or NULL with
 * bias_bits 16 (int16, the reference's type) or 32 (int32, widened exactly as
 * src/int16_ops.cpp:163-167 does on the CPU path), out [n, co, oh, ow].
 * groups == 1, stride 1 and ci*kh*kw <= 32768 run on the tcgen05 tensor cores;
 * other geometries use the direct int64 kernel (as the reference does). */
int ufb_conv2d(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh, int kw,
               const void* bias, int bias_bits, int stride_h, int stride_w, int pad_h, int pad_w, int groups,
               int16_t* out, void* stream);

/* uf_conv_generic (include/uf/cuda_ops.hpp:13-15): same contract, always the
 * direct int64 kernel (no tensor cores). */
int ufb_conv2d_generic(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh,
                       int kw, const void* bias, int bias_bits, int stride_h, int stride_w, int pad_h, int pad_w,
                       int groups, int16_t* out, void* stream);

/* uf_conv_baseline (include/uf/cuda_ops.hpp:16-18): same contract; the
 * tensor-core path whenever the geometry allows it. */
int ufb_conv2d_baseline(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh,
                        int kw, const void* bias, int bias_bits, int stride_h, int stride_w, int pad_h, int pad_w,
                        int groups, int16_t* out, void* stream);

/* uf_add (include/uf/cuda_ops.hpp:19): out = sat(sum of 2..4 tensors). */
int ufb_add(int count, const int16_t* const* values, int64_t numel, int16_t* out, void* stream);

/* uf_mul (include/uf/cuda_ops.hpp:20): out = sat(rna(x * scale / 512)); both
 * 4-D, every scale extent 1 or equal to x's (broadcast). */
int ufb_mul(const int16_t* x, const int64_t* x_shape, const int16_t* scale, const int64_t* scale_shape,
            int16_t* out, void* stream);

/* uf_lut (include/uf/cuda_ops.hpp:21): out = table[x + 32768]; table has 65536
 * entries of table_bits 16 (int16) or 8 (uint8); out has the table's type. */
int ufb_lut(const int16_t* x, int64_t numel, const void* table, int table_bits, void* out, void* stream);

/* uf_bytes (include/uf/cuda_ops.hpp:22): out = rna((2 v - 255) * 512 / 510). */
int ufb_bytes(const uint8_t* x, int64_t numel, int16_t* out, void* stream);

/* uf_wsilu4 (include/uf/cuda_ops.hpp:23): x [n, 4c, h, w] -> out [n, c, h, w],
 * out[:, k] = sat(sum_{j<4} table[x[:, 4k + j] + 32768]). */
int ufb_wsilu4(const int16_t* x, int n, int c4, int h, int w, const int16_t* table, int16_t* out, void* stream);

/* Fixed-point backward bilinear warp (no reference counterpart: the
 * reference's only warp is the float DCVC-FM kernel block_mc_forward,
 * src/dcvc_fm_motion.cu:29-111, which no build target compiles).
 * feature [n, c, h, w] int16, flow [n, 2, h, w] int16 in Q9 pixels (x, y),
 * border clamp, out = sat(rna(sum of Q18 bilinear weights * taps / 2^18)). */
int ufb_warp(const int16_t* feature, const int16_t* flow, int n, int c, int h, int w, int16_t* out,
             void* stream);

/* ---------------------------------------------------------------------------
 * Split-layout operators.  The engine keeps activations in HBM as "split
 * NHWC": per pixel, a row of 2 * pitch bytes holding the low bytes (u8) of its
 * channels followed by their high bytes (s8); value = lo + 256 * hi.  pitch
 * and any channel offset are multiples of 16.  Callers that keep activations
 * resident in this layout avoid the NCHW conversions of ufb_conv2d.
 * ------------------------------------------------------------------------- */

/* NCHW int16 -> split (pixel_unshuffle(factor) fused; factor 1 = layout only).
 * out holds n x (h/f) x (w/f) pixels of c*f*f channels with row pitch `pitch`. */
int ufb_to_split(const int16_t* x, int n, int c, int h, int w, int factor, uint8_t* out, int pitch, void* stream);

/* split -> NCHW int16 (pixel_shuffle(factor) fused).  x holds n x h x w pixels
 * of c channels; out is [n, c/(f*f), h*f, w*f]. */
int ufb_from_split(const uint8_t* x, int n, int c, int h, int w, int pitch, int factor, int16_t* out,
                   void* stream);

/* Bytes of the prepared weight planes for a [co, ci, kh, kw] convolution. */
int64_t ufb_weight_bytes(int co, int ci, int kh, int kw);

/* Prepare int16 [co, ci, kh, kw] weights (device) into tensor-core planes
 * (device, ufb_weight_bytes() bytes). */
int ufb_prepare_weights(const int16_t* weight, int co, int ci, int kh, int kw, uint8_t* planes, void* stream);

/* uf_conv on split activations with prepared weights: stride 1, zero padding
 * (pad_h, pad_w), groups 1, ci*kh*kw <= 32768.  Uses no scratch memory. */
int ufb_conv2d_split(const uint8_t* x, int n, int ci, int h, int w, int x_pitch, const uint8_t* planes, int co,
                     int kh, int kw, const void* bias, int bias_bits, int pad_h, int pad_w, uint8_t* out,
                     int out_pitch, void* stream);

/* Measurement utility (no reference counterpart): launches `ctas` CTAs that
 * each issue `iters` x 4 dense tcgen05 kind::i8 M=128 N=256 K=32 MMAs from
 * resident shared-memory tiles; *int8_ops receives the operation count
 * (2 per multiply-add).  The caller times the launch on `stream` to obtain
 * the int8 tensor-pipe peak used as the convolution roofline. */
int ufb_probe_i8_peak(int iters, int ctas, void* stream, int64_t* int8_ops);

#ifdef __cplusplus
}
#endif

#endif /* UF_B200_H */
