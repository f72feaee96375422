// Launch interfaces of the per-layer kernels (layers.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace qdec {

struct DeltaArgs {
    float* S;                 // [n_v][dk][dv] committed recurrent state
    const float* conved;      // [t][conv_dim] conv + SiLU output
    const float* alpha;       // [t][n_v] ssm_alpha projection
    const float* beta;        // [t][n_v] ssm_beta projection
    const float* z;           // [t][n_v * dv] attn_gate projection
    const float* ssm_a;       // [n_v]
    const float* dt_bias;     // [n_v]
    const float* norm_w;      // [dv]
    float* heads;             // [t][n_v * dv] output
    float* pend_decay;        // [max_t][n_v]
    float* pend_k;            // [max_t][n_v][dk]
    float* pend_delta;        // [max_t][n_v][dv]
    const int* keep_prev;     // device int: pending rows of the previous call to commit (null: 0)
    int t, max_t, n_k, n_v, dk, dv, kd, conv_dim;
    float eps;
    // optional (t <= 8, hid <= 5120): the F32 ssm_alpha / ssm_beta rows [n_v][hid] and the normed rows [t][hid];
    // when set, the kernel computes alpha and beta itself instead of reading them
    const float* w_alpha;
    const float* w_beta;
    const float* xn;
    int hid;
    // optional: the head outputs quantised by this kernel for the out projection -- into the Q8_K image (a
    // 256-value block spans 256 / dv heads: the block's last head to finish quantises it, blk_cnt holding one
    // zeroed counter per block) and / or the Q8_0 image (32-value blocks inside each head)
    uint8_t* img_q8k;
    uint8_t* img_q80;
    unsigned* blk_cnt;
};

struct QkArgs {
    const float* qg;          // [t][n_head][2][hd]: q then gate per head
    const float* k;           // [t][n_kv * hd]
    const float* v;           // [t][n_kv * hd]
    const float* q_norm;      // [hd]
    const float* k_norm;      // [hd]
    const float* cos;         // [max_pos][rope_dim]
    const float* sin;         // [max_pos][rope_dim]
    const int* pos;           // device int: position of row 0
    float* q_out;             // [t][n_head * hd]
    float* gate_out;          // [t][n_head * hd]
    float* k_cache;           // [max_pos][n_kv][hd]
    float* v_cache;
    int n_head, n_kv, head_dim, rope_dim;
    float eps;
};

struct AttnArgs {
    const float* q;           // [t][n_head * hd] normed, roped
    const float* gate;        // [t][n_head * hd]
    const float* k_cache;
    const float* v_cache;
    const int* pos;           // device int: position of row 0 (row i attends to 0..pos+i)
    float* out;               // [t][n_head * hd]
    int n_head, n_kv, head_dim, max_len;
    float scaling;
    float* scores;            // scratch [t][n_head][max_len rounded up to 4] (null: the single-kernel path)
};

cudaError_t launch_resid_norm_quant(const float* a, const float* b, float* h_out, const float* w, float eps, int n, int rows,
                                    float* y_out, uint8_t* q8k_out, uint8_t* q80_out, cudaStream_t s);
cudaError_t launch_rmsnorm_rows(const float* x, int x_ld, const float* w, float eps, int n, int rows, float* y, int y_ld,
                               cudaStream_t s);
cudaError_t launch_swiglu_quant(const float* g, const float* u, int n, int rows, float* h_out, uint8_t* q8k_out,
                                uint8_t* q80_out, cudaStream_t s);
cudaError_t launch_quant_rows(const float* x, int n, int rows, uint8_t* q8k_out, uint8_t* q80_out, cudaStream_t s);
cudaError_t launch_conv_step(float* state, const float* w, int K, int channels, const float* x, int t, float* out,
                             float* pend_x, const int* keep_prev, int max_t, cudaStream_t s);
// The head shapes the device kernels are built for (the Qwen3.8 family's): DeltaNet K heads of 64 or 128 with V
// heads of 32..128 in steps of 32; attention heads of 64..256 in steps of 64.  A model outside them is refused at
// load time.
inline bool deltanet_dims_supported(int dk, int dv) { return (dk == 64 || dk == 128) && dv % 32 == 0 && dv >= 32 && dv <= 128; }
inline bool attention_dims_supported(int head_dim) { return head_dim % 64 == 0 && head_dim >= 64 && head_dim <= 256; }
cudaError_t launch_deltanet_heads(const DeltaArgs& a, cudaStream_t s);
cudaError_t launch_qk_norm_rope(const QkArgs& a, int t, cudaStream_t s);
cudaError_t launch_attention(const AttnArgs& a, int t, cudaStream_t s);
// scratch: argmax_scratch_bytes(n, rows) bytes, zero-filled once before the first use (launches keep it so).
size_t argmax_scratch_bytes(int n, int rows);
cudaError_t launch_argmax(const float* x, int n, int rows, int32_t* out, void* scratch, cudaStream_t s);
// a tensor-parallel rank's slice [base, base + n) of each row: {float value, int global index} at pairs + 16 * row
// (the seed element 0 only when `seed`, i.e. on rank 0)
cudaError_t launch_argmax_pairs(const float* x, int n, int rows, uint8_t* pairs, int base, bool seed, void* scratch,
                                cudaStream_t s);

}  // namespace qdec
