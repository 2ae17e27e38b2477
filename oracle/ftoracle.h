/* ftoracle.h -- CPU restatement of the reference's dequant-matmul path.
 * TEST INFRASTRUCTURE ONLY (checker and "port" CPU baseline); the product
 * library never includes or links this.  See ftoracle.c for citations. */
#ifndef FTORACLE_H
#define FTORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* Type ids: the reference's ft::DType values (ft/include/ft/types.h:20-27)
 * plus the GGUF ids of the two K-quants the reference lacks. */
enum { FTOR_F32 = 0, FTOR_F16 = 1, FTOR_Q4_0 = 2, FTOR_Q4_1 = 3, FTOR_Q8_0 = 8,
       FTOR_Q4_K = 12, FTOR_Q6_K = 14, FTOR_BF16 = 30 };

float ftor_half_to_float(uint16_t h);
uint16_t ftor_float_to_half(float f);
int64_t ftor_block_elems(int dtype);
int64_t ftor_block_bytes(int dtype);
int64_t ftor_row_bytes(int dtype, int64_t n_cols);
int ftor_dequant_row(float* dst, const uint8_t* src, int dtype, int64_t n);
float ftor_dot_row_f32(const float* x, const uint8_t* w, int dtype, int64_t n);
int ftor_matmul(const float* x, int64_t M, int64_t K, const uint8_t* W, int dtype,
                int64_t N, int64_t row_stride, float* y, int threads);
int ftor_expert_chunk(const float* x, float* out, const uint8_t* gate, const uint8_t* up,
                      const uint8_t* down, int dtype, int64_t M, int64_t K, int64_t IC,
                      int64_t gu_stride, int64_t dn_stride, int threads);
int ftor_matmul_down_axpy(const float* x, int64_t M, int64_t n_in, const uint8_t* W, int dtype,
                          int64_t N, int64_t row_stride, float* y, int threads);
int ftor_expert_ffn(const float* x, float* out, const uint8_t* gate, const uint8_t* up,
                    const uint8_t* down, int dtype, int64_t M, int64_t K, int64_t n_ff,
                    int64_t gu_stride, int64_t dn_stride, int threads);
int ftor_route_topk(const float* logits, const float* bias, int64_t T, int64_t E, int64_t U,
                    int32_t* idx, float* w);
int ftor_moe_ffn(const float* x, const float* logits, int64_t T, int64_t K, int64_t n_ff,
                 int64_t E, int64_t U, const uint8_t* gate_exps, const uint8_t* up_exps,
                 const uint8_t* down_exps, int dtype, float* out, int threads);
int ftor_attention(const float* q, int64_t M, int64_t n_head, int64_t n_head_kv,
                   int64_t head_dim, const float* k_cache, const float* v_cache, int64_t base,
                   const float* k_blk, const float* v_blk, float* out, int threads);
void ftor_rope_vec(float* v, int64_t hd, int64_t pos, double theta, int neox);
int ftor_rope(float* x, int64_t M, int64_t heads, int64_t hd, int64_t base, double theta,
              int neox);

#ifdef __cplusplus
}
#endif
#endif
