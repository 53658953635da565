/* TEST INFRASTRUCTURE ONLY: CPU restatement of the reference INT16 arithmetic
 * (contract "uf-int16-q9-w13-acc64-rna-sat-v1").  Only tests/, the smoke check
 * and the bench's CPU arm may load it; the product library never does.
 * All tensors are dense NCHW; every function returns 0 or a negative error. */
#ifndef UF_ORACLE_H
#define UF_ORACLE_H
#include <stdint.h>

int64_t ufo_divide_round(int64_t value, int64_t denominator);
int16_t ufo_saturate(int64_t value);

int ufo_conv2d(const int16_t* x, int64_t n, int64_t ci, int64_t h, int64_t w,
               const int16_t* weight, int64_t co, int64_t kh, int64_t kw,
               const void* bias, int bias_bits, int64_t sh, int64_t sw, int64_t ph,
               int64_t pw, int64_t groups, int16_t* out);
int ufo_add(int count, const int16_t* const* values, int64_t numel, int16_t* out);
int ufo_multiply(const int16_t* x, const int64_t* xs, const int16_t* scale, const int64_t* ss,
                 int16_t* out);
int ufo_lookup_i16(const int16_t* x, int64_t numel, const int16_t* table, int16_t* out);
int ufo_lookup_u8(const int16_t* x, int64_t numel, const uint8_t* table, uint8_t* out);
int ufo_wsilu4(const int16_t* x, int64_t n, int64_t c4, int64_t hw, const int16_t* table,
               int16_t* out);
int ufo_from_bytes(const uint8_t* x, int64_t numel, int16_t* out);
int ufo_symbols(const int16_t* x, int64_t numel, int8_t* out);
int ufo_from_symbols(const int8_t* x, int64_t numel, int16_t* out);
int ufo_reciprocal(const int16_t* x, int64_t numel, int16_t* out);
int ufo_pixel_shuffle(const int16_t* x, int64_t n, int64_t c, int64_t h, int64_t w,
                      int64_t factor, int unshuffle, int16_t* out);
int ufo_raw_frame(const int16_t* frame, int64_t h, int64_t w, int64_t height, int64_t width,
                  uint8_t* out);
int ufo_warp(const int16_t* feature, const int16_t* flow, int64_t n, int64_t c, int64_t h,
             int64_t w, int16_t* out);
int ufo_warp_float(const int16_t* feature, const int16_t* flow, int64_t n, int64_t c, int64_t h,
                   int64_t w, float* out);

#endif
