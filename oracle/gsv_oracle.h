/* gsv_oracle.h -- test-infrastructure CPU restatement of the gpt-sovits-rs
 * SoVITS v2 Generator.  Only tests/, the smoke check and the CPU-baseline leg
 * of bench.py may use it; the product never does. */
#ifndef GSV_ORACLE_H
#define GSV_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  const char* name;   /* safetensors key, e.g. "dec.ups.0.weight_v" */
  const float* data;  /* host fp32, contiguous */
  int ndim;
  int64_t shape[4];
} gsvo_tensor;

const char* gsvo_last_error(void);
void gsvo_leaky_relu(float* x, int64_t n, float slope);
void gsvo_weight_norm(const float* v, const float* g, int O, int I, int K, float* w);
int gsvo_conv1d(const float* x, int B, int Cin, int L, const float* w, int Cout, int K, int pad,
                int dil, const float* bias, float* y, int acc64);
int gsvo_conv_transpose1d(const float* x, int B, int Cin, int L, const float* w, int Cout, int K,
                          int stride, int pad, const float* bias, float* y, int acc64);
int gsvo_decoder_forward(const gsvo_tensor* ts, int n_tensors, const float* z, const float* g,
                         int B, int T0, float* wav, float** taps, int acc64, int nthreads);
/* Flow inverse (src/models/sovits_flow.rs:341-415, reverse = true) followed by
 * z * y_mask (src/models/sovits.rs:394): z_p, z [B, C, T0]; g [B, gin, 1] or
 * NULL; lengths [B] or NULL.  prefix is the state-dict prefix ("flow.flows"). */
int gsvo_flow_inverse(const gsvo_tensor* ts, int n_tensors, const char* prefix, const float* z_p,
                      const float* g, const int* lengths, int B, int T0, float* z, int acc64,
                      int nthreads);

/* EncP elementwise chains (src/models/sovits_encp.rs), see gsv_oracle.c. */
int gsvo_layer_norm(const float* x, const float* y, const float* gamma, const float* beta, int B, int C,
                    int T, float eps, const int* lengths, float* out);
int gsvo_encp_ffn(const float* x, int B, int C, int T, const float* w1, const float* b1, int F, int k1,
                  const float* w2, const float* b2, int k2, const float* gamma, const float* beta,
                  const int* lengths, float* out, int acc64);
int gsvo_interpolate(const float* x, int64_t rows, int T, int T_out, float* out);
int gsvo_encp_project(const float* y, int B, int C, int T, const float* w, const float* bias, int Co2,
                      const int* lengths, const float* noise, float noise_scale, float* m, float* logs,
                      float* z_p, int acc64);

#ifdef __cplusplus
}
#endif
#endif
