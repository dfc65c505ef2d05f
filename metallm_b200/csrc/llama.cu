// llama.cu -- the decode runner: LlamaRunner (MetalLM/Backend/LlamaRunner.swift)
// on this library's kernels.
//
// The reference encodes every decode step op by op: a blit for the
// embedding row, then per layer RMSNorm, three MPS GEMMs on fp16 weights
// dequantized at load, RoPE, a KV-cache blit, repeat-KV plus 32 per-head
// GEMM / softmax / GEMM triples, the output projection, a residual add,
// RMSNorm, gate/up GEMMs, SiLU, multiply, the down GEMM and a residual add;
// then the final norm, the output GEMM and a CPU argmax
// (LlamaRunner.swift:320-1210, ContentView.swift:124-146).
//
// Here the runner owns the weights in Q4_K GGUF layout, with wq/wk/wv and
// w_gate/w_up stored as one row-concatenated matrix each so that they run as
// one GEMV; residual adds are fused into the GEMVs that produce them; RoPE
// and the cache append are one kernel; attention is one split-sequence
// kernel pair over the fp16 cache; the RMSNorms and the SiLU-gated product
// are computed inside the x staging of the GEMVs that consume them.  A
// decode step is 6 launches per layer plus 4.  The hidden state stays fp32 between layers (the reference keeps
// fp16); GEMV inputs are fp16 as in the reference, the SiLU-gated product
// with a power-of-two scale per 32 elements (a plain fp16 store overflows
// there on large activations; the reference's does).  Token, position and
// step counter live in device memory, so a step is captured once as a CUDA
// graph and replayed for every generated token.  The prompt runs batched:
// per layer, RMSNorm rows, the tensor-core Q4_K GEMM for the fused QKV, RoPE
// with the cache append, causal attention over the cache, the GEMM for the
// output projection (residual added), RMSNorm, the gate/up GEMM, SiLU-gated
// product and the down GEMM (residual added), in chunks of up to 1024 tokens.
//
// Tensor parallelism (when the context has an NCCL group, mlm_tp_init): each
// rank holds its share of the heads (QKV rows, KV cache, attention), of the
// FFN rows (gate/up) and of the vocabulary (output head), and the matching
// input columns of the output and down projections, which therefore produce
// partial sums: rank 0 adds the residual into its partial and one NCCL sum
// all-reduce lands the new hidden state on every rank, twice per layer.  The
// greedy token is the maximum of the ranks' argmax keys (one 8-byte
// all-gather).  Everything stays on the context's stream, so the sharded
// decode step is captured as one CUDA graph like the single-GPU one.
#include <cuda_runtime.h>

#include <algorithm>
#include <new>
#include <vector>

#include "mlm_device.cuh"
#include "mlm_internal.h"

namespace mlm {
namespace {

struct LayerBuf {
  float *attn_norm, *ffn_norm;
  // Q4_K, except wv and down, which are Q6_K when v_type / down_type say so
  // (Q4_K_M files); a Q4_K wv is the last rows of qkv, a Q6_K one separate
  uint8_t *qkv, *wo, *gu, *down, *wv6 = nullptr;
  int v_type = MLM_TYPE_Q4_K, down_type = MLM_TYPE_Q4_K;
  __half *kc, *vc;
};

// device step state
enum { kToken = 0, kPos = 1, kStep = 2, kStateInts = 4 };

__global__ void set_state_kernel(int *st, int token, int pos, int step) {
  st[kToken] = token;
  st[kPos] = pos;
  st[kStep] = step;
}

// after the argmax of a step: record its token, move to the next position
__global__ void advance_kernel(int *st, int32_t *tokens) {
  pdl_wait_then_release();
  tokens[st[kStep]] = st[kToken];
  st[kStep] += 1;
  st[kPos] += 1;
}

// the same for a batch of sequences: gen[step][b] = tok[b], positions + 1
__global__ void advance_batch_kernel(int *st, int *pos, const int32_t *tok, int32_t *gen,
                                     int batch) {
  pdl_wait_then_release();
  const int step = st[kStep];
  for (int b = threadIdx.x; b < batch; b += blockDim.x) {
    gen[(size_t)step * batch + b] = tok[b];
    pos[b] += 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) st[kStep] = step + 1;
}

inline size_t q4k_row_bytes(int cols) { return (size_t)(cols / kQK) * kBlockBytes; }
constexpr int kQ6BlockBytes = 210;
inline size_t q6k_row_bytes(int cols) { return (size_t)(cols / kQK) * kQ6BlockBytes; }
inline size_t row_bytes(int type, int cols) {
  return type == MLM_TYPE_Q6_K ? q6k_row_bytes(cols) : q4k_row_bytes(cols);
}

}  // namespace
}  // namespace mlm

using namespace mlm;

struct mlm_llama {
  mlm_ctx *ctx = nullptr;
  mlm_llama_config cfg{};
  int pos = 0;
  std::vector<LayerBuf> layers;
  __half *tok_embd = nullptr;
  float *out_norm = nullptr;
  uint8_t *output = nullptr;
  int output_type = MLM_TYPE_Q4_K;
  void *q6_scratch = nullptr;  // bf16 copy of a Q6_K weight for the GEMMs
  float *rope_freqs = nullptr;
  // activations of one step
  float *hidden = nullptr, *qkv_out = nullptr, *gu_out = nullptr, *logits = nullptr;
  __half *attn_out = nullptr;
  __half *ffn_h = nullptr;  // silu(gate) * up as scaled fp16, from the gate/up GEMV
  float *ffn_h_scale = nullptr;
  int *state = nullptr;
  int32_t *gen_tokens = nullptr;  // [max_seq] tokens of the captured greedy loop
  // batched prompt pass: activations of up to pf_chunk tokens
  int pf_chunk = 0;
  float *pf_hidden = nullptr, *pf_qkv = nullptr, *pf_gu = nullptr;
  float *pf_tmp = nullptr;  // q/k rows and v rows apart when V is Q6_K
  void *pf_x = nullptr, *pf_q16 = nullptr, *pf_attn = nullptr;  // bf16 / fp16 / bf16
  int32_t *pf_tokens = nullptr;
  cudaGraph_t step_graph = nullptr;
  cudaGraphExec_t step_exec = nullptr;
  std::vector<void *> allocs;
  // tensor parallelism: this rank's share (tp == 1 and !tp_on: one GPU)
  bool tp_on = false;
  int tp = 1, rank = 0;
  float *part = nullptr, *pf_part = nullptr, *logits_l = nullptr;  // partial sums, local logits
  unsigned long long *key_l = nullptr, *keys = nullptr;            // argmax keys: own, all ranks
  // a batch of sequences (mlm_llama_create_batch): sequence b's KV caches
  // start b * seq_elems() elements into each layer's; `pos` is sequence 0's
  // position (and, inside mlm_llama_prefill_seq, that of the sequence cur)
  int batch = 1, cur = 0;
  std::vector<int> seq_pos;                     // positions of sequences 1.. (0: pos)
  int *pos_b = nullptr;                         // device positions [batch]
  int32_t *tok_b = nullptr;                     // device tokens [batch]
  int32_t *gen_b = nullptr;                     // [max_seq][batch] greedy tokens
  float *b_logits = nullptr;                    // [batch][vocab / tp]
  unsigned long long *b_keys_l = nullptr, *b_keys = nullptr;  // [batch], [tp][batch]
  cudaGraph_t bstep_graph = nullptr;
  cudaGraphExec_t bstep_exec = nullptr;

  size_t seq_elems() const { return (size_t)cfg.max_seq * kvdim(); }
  int position(int b) const { return b == 0 ? pos : seq_pos[b]; }

  int nh() const { return cfg.n_heads / tp; }
  int nkv() const { return cfg.n_kv_heads / tp; }
  int ffn() const { return cfg.ffn_dim / tp; }
  int vocab_l() const { return cfg.vocab / tp; }
  int qdim() const { return nh() * cfg.head_dim; }
  int kvdim() const { return nkv() * cfg.head_dim; }
  int qkv_rows() const { return qdim() + 2 * kvdim(); }
  // rows of layer l's Q4_K QKV matrix (q, k and, when V is Q4_K, v)
  int qkv4_rows(const LayerBuf &L) const {
    return L.v_type == MLM_TYPE_Q6_K ? qdim() + kvdim() : qkv_rows();
  }

  template <class T>
  int alloc(T **p, size_t bytes) {
    void *q = nullptr;
    if (cudaMalloc(&q, bytes ? bytes : 16) != cudaSuccess) {
      cudaGetLastError();
      return set_error(ctx, MLM_ERR_ALLOC, "mlm_llama_create: cudaMalloc(%zu) failed", bytes);
    }
    allocs.push_back(q);
    *p = reinterpret_cast<T *>(q);
    return MLM_OK;
  }

  int gemv(const uint8_t *W, int rows, int cols, const GemvInput &in, float *y, const float *res) {
    return gemv_launch(ctx, W, rows, cols, in, y, res, ctx->gemv_partials, ctx->gemv_counters,
                       ctx->gemv_max_ctas, ctx->gemv_max_tiles, ctx->stream);
  }
  GemvInput normed(const float *h, const float *w) const {
    GemvInput in;
    in.mode = GemvInput::kRmsNorm;
    in.a = h;
    in.b = w;
    in.eps = cfg.rms_eps;
    return in;
  }

  // one decoder layer at the device position state[kPos]
  int layer(int l, float *h) {
    const LayerBuf &L = layers[l];
    const mlm_llama_config &c = cfg;
    cudaStream_t s = ctx->stream;
    int st;
    // RMSNorm runs inside the GEMV's x staging
    if ((st = gemv(L.qkv, qkv4_rows(L), c.dim, normed(h, L.attn_norm), qkv_out, nullptr)))
      return st;
    if (L.v_type == MLM_TYPE_Q6_K &&
        (st = q6k_gemv_launch(ctx, L.wv6, kvdim(), c.dim, normed(h, L.attn_norm),
                              qkv_out + qdim() + kvdim(), nullptr, s)))
      return st;
    // RoPE of q and k, the KV append and the attention in one launch
    if ((st = attn_rope_decode_launch(ctx, qkv_out, rope_freqs, c.rope, nh(), nkv(), c.head_dim,
                                      c.max_seq, L.kc, L.vc, attn_out, s, state + kPos)))
      return st;
    if ((st = row_parallel(L.wo, qdim(), gemv_half(attn_out), h))) return st;  // + residual
    // the gate/up GEMV's epilogue forms the SiLU-gated product once per
    // element, as fp16 with per-32 power-of-two scales (it exceeds the fp16
    // range on large activations); the down projection stages it as is
    GemvPair pair;
    pair.h_f16 = ffn_h;
    pair.h_scale = ffn_h_scale;
    pair.counters = ctx->gemv_counters + ctx->gemv_max_tiles;
    if ((st = gemv_launch(ctx, L.gu, 2 * ffn(), c.dim, normed(h, L.ffn_norm), gu_out, nullptr,
                          ctx->gemv_partials, ctx->gemv_counters, ctx->gemv_max_ctas,
                          ctx->gemv_max_tiles, s, &pair)))
      return st;
    return row_parallel(L.down, ffn(), gemv_half(ffn_h, ffn_h_scale), h, L.down_type);
  }

  // a decode GEMV on a weight of either type
  int gemv_t(int type, const uint8_t *W, int rows, int cols, const GemvInput &in, float *y,
             const float *res) {
    if (type == MLM_TYPE_Q6_K) return q6k_gemv_launch(ctx, W, rows, cols, in, y, res, ctx->stream);
    return gemv(W, rows, cols, in, y, res);
  }

  // h += W x for a projection whose input columns are split over the ranks:
  // in place on one GPU; with TP, rank 0's partial carries the residual and
  // the sum all-reduce writes h on every rank
  int row_parallel(const uint8_t *W, int cols, const GemvInput &in, float *h,
                   int type = MLM_TYPE_Q4_K) {
    if (!tp_on) return gemv_t(type, W, cfg.dim, cols, in, h, h);
    int st = gemv_t(type, W, cfg.dim, cols, in, part, rank == 0 ? h : nullptr);
    if (st != MLM_OK) return st;
    return tp_allreduce_sum(ctx, part, h, cfg.dim, ctx->stream);
  }

  // final norm, the output GEMV and the greedy token into state[kToken];
  // the full logits also land in lg_out when it is given
  int head(const float *h, float *lg_out) {
    int st;
    if (!tp_on) {
      float *lg = lg_out ? lg_out : logits;
      if ((st = gemv_t(output_type, output, cfg.vocab, cfg.dim, normed(h, out_norm), lg, nullptr)))
        return st;
      return argmax_launch(ctx, lg, cfg.vocab, state + kToken, ctx->stream);
    }
    if ((st = gemv_t(output_type, output, vocab_l(), cfg.dim, normed(h, out_norm), logits_l,
                     nullptr)))
      return st;
    if ((st = argmax_key_launch(ctx, logits_l, vocab_l(), rank * vocab_l(), key_l, ctx->stream)))
      return st;
    if ((st = tp_allgather_bytes(ctx, key_l, keys, sizeof(unsigned long long), ctx->stream)))
      return st;
    if ((st = argmax_keys_launch(ctx, keys, tp, state + kToken, ctx->stream))) return st;
    if (lg_out)
      return tp_allgather_bytes(ctx, logits_l, lg_out, sizeof(float) * vocab_l(), ctx->stream);
    return MLM_OK;
  }

  // embedding of state[kToken], all layers; then, when `with_head`, the
  // final norm, the output GEMV (logits into lg when given) and the argmax
  // into state[kToken]
  int step(bool with_head, float *lg) {
    int st;
    if ((st = embed_launch(ctx, tok_embd, cfg.vocab, cfg.dim, state + kToken, hidden,
                           ctx->stream)))
      return st;
    for (int l = 0; l < cfg.n_layers; ++l)
      if ((st = layer(l, hidden))) return st;
    if (!with_head) return MLM_OK;
    return head(hidden, lg);
  }

  // T prompt tokens (device ids in pf_tokens) at positions pos .. pos+T-1:
  // every layer on the tensor-core GEMM; leaves the hidden rows in pf_hidden
  int prefill_chunk(int T) {
    const mlm_llama_config &c = cfg;
    cudaStream_t s = ctx->stream;
    int st;
    if ((st = embed_rows_launch(ctx, tok_embd, c.vocab, c.dim, pf_tokens, T, pf_hidden, s))) return st;
    for (int l = 0; l < c.n_layers; ++l) {
      const LayerBuf &L = layers[l];
      const bool zq = T <= 8 && L.v_type != MLM_TYPE_Q6_K;  // batched GEMV: accumulates
      if ((st = rmsnorm_rows_bf16_launch(ctx, pf_hidden, L.attn_norm, pf_x, T, c.dim, c.rms_eps, s,
                                         zq ? pf_qkv : nullptr, (size_t)T * qkv_rows())))
        return st;
      if ((st = qkv_rows_linear(L, pf_x, T, zq))) return st;
      __half *kc = L.kc + cur * seq_elems(), *vc = L.vc + cur * seq_elems();
      if ((st = rope_kv_rows_launch(ctx, pf_qkv, rope_freqs, c.rope, nh(), nkv(), c.head_dim, pos,
                                    T, pf_q16, kc, vc, s)))
        return st;
      if ((st = attn_prefill_launch(ctx, pf_q16, kc, vc, pos, T, nh(), nkv(), c.head_dim,
                                    pf_attn, s)))
        return st;
      if ((st = row_parallel_rows(L.wo, qdim(), pf_attn, T))) return st;
      if ((st = rmsnorm_rows_bf16_launch(ctx, pf_hidden, L.ffn_norm, pf_x, T, c.dim, c.rms_eps, s,
                                         T <= 8 ? pf_gu : nullptr, (size_t)T * 2 * ffn())))
        return st;
      if ((st = linear(L.gu, 2 * ffn(), c.dim, pf_x, T, pf_gu, nullptr, T <= 8))) return st;
      if ((st = swiglu_rows_bf16_launch(ctx, pf_gu, ffn(), T, pf_x, s))) return st;
      if ((st = row_parallel_rows(L.down, ffn(), pf_x, T, L.down_type))) return st;
    }
    return MLM_OK;
  }

  // pf_qkv = X Wqkv^T over T rows [T][q | k | v]: one Q4_K linear, or the
  // Q4_K q/k rows and the Q6_K v rows written beside them
  int qkv_rows_linear(const LayerBuf &L, const void *x, int T, bool y_zeroed = false) {
    if (L.v_type != MLM_TYPE_Q6_K)
      return linear(L.qkv, qkv_rows(), cfg.dim, x, T, pf_qkv, nullptr, y_zeroed);
    const int r4 = qkv4_rows(L);
    int st = linear(L.qkv, r4, cfg.dim, x, T, pf_tmp, nullptr);
    if (st != MLM_OK) return st;
    if ((st = linear_q6(L.wv6, kvdim(), cfg.dim, x, T, pf_tmp + (size_t)T * r4, nullptr,
                        [&](int t) { return rms_row(t, L.attn_norm); })))
      return st;
    return interleave_rows_launch(ctx, pf_tmp, r4, pf_tmp + (size_t)T * r4, kvdim(), T, pf_qkv,
                                  ctx->stream);
  }

  // one decode step of every sequence of the batch (token tok_b[b] at
  // position pos_b[b]): the prompt pass's row kernels and tensor-core GEMMs
  // over the batch's B rows, attention per sequence over its own cache; the
  // greedy tokens land in tok_b; logits (all rows, [B][vocab]) in lg_out
  // when it is given
  int step_batch(float *lg_out) {
    const mlm_llama_config &c = cfg;
    cudaStream_t s = ctx->stream;
    const int B = batch;
    int st;
    if ((st = embed_rows_launch(ctx, tok_embd, c.vocab, c.dim, tok_b, B, pf_hidden, s))) return st;
    for (int l = 0; l < c.n_layers; ++l) {
      const LayerBuf &L = layers[l];
      const bool zq = L.v_type != MLM_TYPE_Q6_K;  // the batched GEMV accumulates into pf_qkv
      if ((st = rmsnorm_rows_bf16_launch(ctx, pf_hidden, L.attn_norm, pf_x, B, c.dim, c.rms_eps, s,
                                         zq ? pf_qkv : nullptr, (size_t)B * qkv_rows())))
        return st;
      if ((st = qkv_rows_linear(L, pf_x, B, zq))) return st;
      // RoPE of q and k, the KV append and the attention of every sequence
      if ((st = attn_rope_decode_batch_launch(ctx, pf_qkv, qkv_rows(), rope_freqs, c.rope, nh(),
                                              nkv(), c.head_dim, c.max_seq, B, seq_elems(),
                                              L.kc, L.vc, pf_attn, s, pos_b)))
        return st;
      if ((st = row_parallel_rows(L.wo, qdim(), pf_attn, B))) return st;
      if ((st = rmsnorm_rows_bf16_launch(ctx, pf_hidden, L.ffn_norm, pf_x, B, c.dim, c.rms_eps, s,
                                         pf_gu, (size_t)B * 2 * ffn())))
        return st;
      if ((st = linear(L.gu, 2 * ffn(), c.dim, pf_x, B, pf_gu, nullptr, true))) return st;
      if ((st = swiglu_rows_bf16_launch(ctx, pf_gu, ffn(), B, pf_x, s))) return st;
      if ((st = row_parallel_rows(L.down, ffn(), pf_x, B, L.down_type))) return st;
    }
    if (output_type == MLM_TYPE_Q6_K) {
      // a Q6_K head: one GEMV per row, RMSNorm in its staging (a bf16 copy
      // of the head would not fit the scratch)
      for (int b = 0; b < B; ++b)
        if ((st = q6k_gemv_launch(ctx, output, vocab_l(), c.dim,
                                  normed(pf_hidden + (size_t)b * c.dim, out_norm),
                                  b_logits + (size_t)b * vocab_l(), nullptr, s)))
          return st;
    } else {
      if ((st = rmsnorm_rows_bf16_launch(ctx, pf_hidden, out_norm, pf_x, B, c.dim, c.rms_eps, s)))
        return st;
      if ((st = linear(output, vocab_l(), c.dim, pf_x, B, b_logits, nullptr))) return st;
    }
    for (int b = 0; b < B; ++b) {
      st = tp_on ? argmax_key_launch(ctx, b_logits + (size_t)b * vocab_l(), vocab_l(),
                                     rank * vocab_l(), b_keys_l + b, s)
                 : argmax_launch(ctx, b_logits + (size_t)b * c.vocab, c.vocab, tok_b + b, s);
      if (st != MLM_OK) return st;
    }
    if (tp_on) {
      if ((st = tp_allgather_bytes(ctx, b_keys_l, b_keys, sizeof(unsigned long long) * B, s)))
        return st;
      if ((st = argmax_keys_rows_launch(ctx, b_keys, tp, B, tok_b, s))) return st;
    }
    if (lg_out) {
      if (!tp_on)
        MLM_CUDA_TRY(ctx, cudaMemcpyAsync(lg_out, b_logits, sizeof(float) * B * c.vocab,
                                          cudaMemcpyDeviceToDevice, s));
      else
        for (int b = 0; b < B; ++b)  // row b: rank r's slice lands at [b][r V/R ..)
          if ((st = tp_allgather_bytes(ctx, b_logits + (size_t)b * vocab_l(),
                                       lg_out + (size_t)b * c.vocab, sizeof(float) * vocab_l(),
                                       s)))
            return st;
    }
    return MLM_OK;
  }

  // Y = X W^T (+ residual) over T token rows of bf16 X: up to 8 rows (a
  // decode batch) stream the weights through the batched GEMV, more through
  // the tensor-core GEMM
  // y_zeroed: y was cleared by the kernel before (the RMSNorm rows feeding
  // this linear), so the batched GEMV needs no memset of its own
  int linear(const uint8_t *W, int rows, int cols, const void *x, int T, float *y,
             const float *res, bool y_zeroed = false) {
    if (T <= 8)
      return gemv_batch_launch(ctx, W, rows, cols, x, T, y, res, ctx->stream, y_zeroed);
    return gemm_launch(ctx, W, rows, cols, x, T, y, res, ctx->stream);
  }
  // A Q6_K weight over T token rows.  Up to 8 rows (a decode batch, a short
  // prompt): one Q6_K GEMV per row with x staged from the fp32 source the
  // single-token step uses (src(t): the RMSNorm or SiLU-gated input of row
  // t), so these rows compute what the decode step computes.  More rows: the
  // bf16 x through the weight's bf16 copy in q6_scratch and the GEMM.
  template <class Src>
  int linear_q6(const uint8_t *W, int rows, int cols, const void *x_bf16, int T, float *y,
                const float *res, Src src) {
    if (T > 8)
      return q6k_gemm_launch(ctx, W, rows, cols, x_bf16, T, y, res, q6_scratch, ctx->stream);
    for (int t = 0; t < T; ++t) {
      int st = q6k_gemv_launch(ctx, W, rows, cols, src(t), y + (size_t)t * rows,
                               res ? res + (size_t)t * rows : nullptr, ctx->stream);
      if (st != MLM_OK) return st;
    }
    return MLM_OK;
  }
  GemvInput rms_row(int t, const float *norm_w) const {
    return normed(pf_hidden + (size_t)t * cfg.dim, norm_w);
  }
  GemvInput swiglu_row(int t) const {
    GemvInput in;
    in.mode = GemvInput::kSwiGLU;
    in.a = pf_gu + (size_t)t * 2 * ffn();
    in.b = in.a + ffn();
    return in;
  }

  // pf_hidden += X W^T over T rows for a projection with split input
  // columns (see row_parallel); a Q6_K one is the down projection
  int row_parallel_rows(const uint8_t *W, int cols, const void *x, int T,
                        int type = MLM_TYPE_Q4_K) {
    auto lin = [&](float *y, const float *res) {
      if (type != MLM_TYPE_Q6_K) return linear(W, cfg.dim, cols, x, T, y, res);
      return linear_q6(W, cfg.dim, cols, x, T, y, res, [&](int t) { return swiglu_row(t); });
    };
    if (!tp_on) return lin(pf_hidden, pf_hidden);
    int st = lin(pf_part, rank == 0 ? pf_hidden : nullptr);
    if (st != MLM_OK) return st;
    return tp_allreduce_sum(ctx, pf_part, pf_hidden, (size_t)T * cfg.dim, ctx->stream);
  }

  int set_state(int token, int p, int stp) {
    set_state_kernel<<<1, 1, 0, ctx->stream>>>(state, token, p, stp);
    return check_launch(ctx, "mlm_llama (state)");
  }

  void destroy() {
    if (step_exec) cudaGraphExecDestroy(step_exec);
    if (step_graph) cudaGraphDestroy(step_graph);
    if (bstep_exec) cudaGraphExecDestroy(bstep_exec);
    if (bstep_graph) cudaGraphDestroy(bstep_graph);
    for (void *p : allocs) cudaFree(p);
    allocs.clear();
  }
};

static bool known_type(int t) { return t == MLM_TYPE_Q4_K || t == MLM_TYPE_Q6_K; }

static int llama_create(mlm_ctx *ctx, const mlm_llama_config *cfg, int batch,
                        const mlm_llama_types *types, mlm_llama **out) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, cfg && out, MLM_ERR_ARG, "mlm_llama_create: null argument");
  *out = nullptr;
  const mlm_llama_config &c = *cfg;
  // tensor types: everything Q4_K unless types says otherwise
  const int out_type = types ? types->output : MLM_TYPE_Q4_K;
  auto v_type = [&](int l) { return types && types->attn_v ? types->attn_v[l] : MLM_TYPE_Q4_K; };
  auto d_type = [&](int l) {
    return types && types->ffn_down ? types->ffn_down[l] : MLM_TYPE_Q4_K;
  };
  MLM_REQUIRE(ctx, batch >= 1 && batch <= 64 && batch <= std::min(c.max_seq, 1024), MLM_ERR_SHAPE,
              "mlm_llama_create_batch: batch %d (1 .. min(64, max_seq))", batch);
  MLM_REQUIRE(ctx, c.n_layers > 0 && c.vocab > 0 && c.max_seq > 0 && c.max_seq <= 8192,
              MLM_ERR_SHAPE, "mlm_llama_create: layers=%d vocab=%d max_seq=%d (max 8192)",
              c.n_layers, c.vocab, c.max_seq);
  MLM_REQUIRE(ctx, c.head_dim == 128 && c.n_heads * c.head_dim == c.dim, MLM_ERR_UNSUPPORTED,
              "mlm_llama_create: head_dim=%d n_heads=%d dim=%d (head_dim 128, n_heads*head_dim "
              "== dim)",
              c.head_dim, c.n_heads, c.dim);
  MLM_REQUIRE(ctx, c.dim % kQK == 0 && c.ffn_dim % kQK == 0, MLM_ERR_SHAPE,
              "mlm_llama_create: dim=%d ffn=%d must be multiples of 256", c.dim, c.ffn_dim);
  MLM_REQUIRE(ctx, c.n_kv_heads > 0 && c.n_heads % c.n_kv_heads == 0, MLM_ERR_SHAPE,
              "mlm_llama_create: %d heads, %d KV heads", c.n_heads, c.n_kv_heads);
  MLM_REQUIRE(ctx, c.rope.n_dims >= 2 && (int)c.rope.n_dims <= c.head_dim, MLM_ERR_SHAPE,
              "mlm_llama_create: rope n_dims=%d", (int)c.rope.n_dims);
  MLM_REQUIRE(ctx, 2 * c.ffn_dim <= ctx->gemv_max_tiles * 32 && c.vocab <= ctx->gemv_max_tiles * 32,
              MLM_ERR_SHAPE, "mlm_llama_create: matrices exceed the GEMV row limit");
  const int tp = ctx->tp_comm ? ctx->tp_size : 1;
  bool any_v6 = false, any_d6 = false;
  MLM_REQUIRE(ctx, known_type(out_type), MLM_ERR_UNSUPPORTED,
              "mlm_llama_create: output type %d (Q4_K %d or Q6_K %d)", out_type, MLM_TYPE_Q4_K,
              MLM_TYPE_Q6_K);
  for (int l = 0; l < c.n_layers; ++l) {
    MLM_REQUIRE(ctx, known_type(v_type(l)) && known_type(d_type(l)), MLM_ERR_UNSUPPORTED,
                "mlm_llama_create: layer %d attn_v type %d / ffn_down type %d (Q4_K %d or Q6_K %d)",
                l, v_type(l), d_type(l), MLM_TYPE_Q4_K, MLM_TYPE_Q6_K);
    any_v6 |= v_type(l) == MLM_TYPE_Q6_K;
    any_d6 |= d_type(l) == MLM_TYPE_Q6_K;
  }
  // the Q6_K decode GEMV reads whole 8-block (2048-column) chunks
  MLM_REQUIRE(ctx,
              ((!any_v6 && out_type != MLM_TYPE_Q6_K) || c.dim % 2048 == 0) &&
                  (!any_d6 || (c.ffn_dim / tp) % 2048 == 0),
              MLM_ERR_UNSUPPORTED,
              "mlm_llama_create: Q6_K tensors need a multiple of 2048 input columns per rank "
              "(dim %d, FFN %d over %d ranks)",
              c.dim, c.ffn_dim, tp);
  if (ctx->tp_comm) {
    // heads, FFN rows and the vocabulary split evenly; the split input
    // columns of the output and down projections stay whole Q4_K blocks
    MLM_REQUIRE(ctx,
                c.n_heads % tp == 0 && c.n_kv_heads % tp == 0 && c.vocab % tp == 0 &&
                    (c.ffn_dim / tp) % kQK == 0 && c.ffn_dim % tp == 0 &&
                    (c.n_heads / tp * c.head_dim) % kQK == 0,
                MLM_ERR_SHAPE,
                "mlm_llama_create: %d ranks do not divide heads %d / KV heads %d / FFN %d / vocab "
                "%d into whole shards",
                tp, c.n_heads, c.n_kv_heads, c.ffn_dim, c.vocab);
  }

  mlm_llama *m = new (std::nothrow) mlm_llama();
  if (!m) return MLM_ERR_ALLOC;
  m->ctx = ctx;
  m->cfg = c;
  m->tp_on = ctx->tp_comm != nullptr;
  m->tp = tp;
  m->rank = ctx->tp_comm ? ctx->tp_rank : 0;
  m->batch = batch;
  m->seq_pos.assign(batch, 0);
  auto fail = [&](int code) {
    m->destroy();
    delete m;
    return code;
  };
  const size_t rb_dim = q4k_row_bytes(c.dim), rb_q = q4k_row_bytes(m->qdim());
  const size_t cache_bytes = (size_t)batch * c.max_seq * m->kvdim() * sizeof(__half);
  m->output_type = out_type;
  m->layers.resize(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    LayerBuf &L = m->layers[l];
    L.v_type = v_type(l);
    L.down_type = d_type(l);
    if (m->alloc(&L.attn_norm, sizeof(float) * c.dim) || m->alloc(&L.ffn_norm, sizeof(float) * c.dim) ||
        m->alloc(&L.qkv, (size_t)m->qkv4_rows(L) * rb_dim) || m->alloc(&L.wo, (size_t)c.dim * rb_q) ||
        m->alloc(&L.gu, (size_t)2 * m->ffn() * rb_dim) ||
        m->alloc(&L.down, (size_t)c.dim * row_bytes(L.down_type, m->ffn())) ||
        (L.v_type == MLM_TYPE_Q6_K &&
         m->alloc(&L.wv6, (size_t)m->kvdim() * q6k_row_bytes(c.dim))) ||
        m->alloc(&L.kc, cache_bytes) || m->alloc(&L.vc, cache_bytes))
      return fail(MLM_ERR_ALLOC);
  }
  // bf16 copy of the largest Q6_K weight the prompt GEMMs read
  const size_t scratch_elems = std::max(any_v6 ? (size_t)m->kvdim() * c.dim : 0,
                                        any_d6 ? (size_t)c.dim * m->ffn() : 0);
  if (scratch_elems && m->alloc(&m->q6_scratch, 2 * scratch_elems)) return fail(MLM_ERR_ALLOC);
  if (m->alloc(&m->tok_embd, (size_t)c.vocab * c.dim * sizeof(__half)) ||
      m->alloc(&m->out_norm, sizeof(float) * c.dim) ||
      m->alloc(&m->output, (size_t)m->vocab_l() * row_bytes(out_type, c.dim)) ||
      m->alloc(&m->rope_freqs, sizeof(float) * (c.head_dim / 2)) ||
      m->alloc(&m->hidden, sizeof(float) * c.dim) ||
      m->alloc(&m->qkv_out, sizeof(float) * m->qkv_rows()) ||
      m->alloc(&m->gu_out, sizeof(float) * 2 * m->ffn()) ||
      m->alloc(&m->logits, sizeof(float) * c.vocab) ||
      m->alloc(&m->attn_out, sizeof(__half) * m->qdim()) ||
      m->alloc(&m->ffn_h, sizeof(__half) * m->ffn()) ||
      m->alloc(&m->ffn_h_scale, sizeof(float) * (m->ffn() / 32)) ||
      m->alloc(&m->state, sizeof(int) * kStateInts) ||
      m->alloc(&m->gen_tokens, sizeof(int32_t) * c.max_seq))
    return fail(MLM_ERR_ALLOC);
  m->pf_chunk = std::min(c.max_seq, 1024);
  {
    const size_t T = m->pf_chunk;
    const size_t xw = std::max(c.dim, m->ffn());
    if (m->alloc(&m->pf_hidden, sizeof(float) * T * c.dim) ||
        m->alloc(&m->pf_qkv, sizeof(float) * T * m->qkv_rows()) ||
        m->alloc(&m->pf_gu, sizeof(float) * T * 2 * m->ffn()) ||
        m->alloc(&m->pf_x, 2 * T * xw) || m->alloc(&m->pf_q16, 2 * T * m->qdim()) ||
        m->alloc(&m->pf_attn, 2 * T * m->qdim()) || m->alloc(&m->pf_tokens, sizeof(int32_t) * T) ||
        (any_v6 && m->alloc(&m->pf_tmp, sizeof(float) * T * m->qkv_rows())))
      return fail(MLM_ERR_ALLOC);
    if (m->alloc(&m->pos_b, sizeof(int) * batch) || m->alloc(&m->tok_b, sizeof(int32_t) * batch) ||
        m->alloc(&m->gen_b, sizeof(int32_t) * c.max_seq * batch) ||
        m->alloc(&m->b_logits, sizeof(float) * batch * m->vocab_l()) ||
        m->alloc(&m->b_keys_l, sizeof(unsigned long long) * batch) ||
        m->alloc(&m->b_keys, sizeof(unsigned long long) * batch * tp))
      return fail(MLM_ERR_ALLOC);
    if (m->tp_on &&
        (m->alloc(&m->part, sizeof(float) * c.dim) ||
         m->alloc(&m->pf_part, sizeof(float) * T * c.dim) ||
         m->alloc(&m->logits_l, sizeof(float) * m->vocab_l()) ||
         m->alloc(&m->key_l, sizeof(unsigned long long)) ||
         m->alloc(&m->keys, sizeof(unsigned long long) * tp)))
      return fail(MLM_ERR_ALLOC);
  }
  if (cudaMemsetAsync(m->state, 0, sizeof(int) * kStateInts, ctx->stream) != cudaSuccess)
    return fail(set_error(ctx, MLM_ERR_CUDA, "mlm_llama_create: memset failed"));
  *out = m;
  return MLM_OK;
}

extern "C" int mlm_llama_create(mlm_ctx *ctx, const mlm_llama_config *cfg, mlm_llama **out) {
  return llama_create(ctx, cfg, 1, nullptr, out);
}

extern "C" int mlm_llama_create_batch(mlm_ctx *ctx, const mlm_llama_config *cfg, int batch,
                                      mlm_llama **out) {
  return llama_create(ctx, cfg, batch, nullptr, out);
}

extern "C" int mlm_llama_create_typed(mlm_ctx *ctx, const mlm_llama_config *cfg, int batch,
                                      const mlm_llama_types *types, mlm_llama **out) {
  return llama_create(ctx, cfg, batch, types, out);
}

extern "C" void mlm_llama_destroy(mlm_llama *m) {
  if (!m) return;
  cudaStreamSynchronize(m->ctx->stream);
  m->destroy();
  delete m;
}

extern "C" int mlm_llama_layer_tensors(mlm_llama *m, int layer, mlm_llama_layer *out) {
  if (!m) return MLM_ERR_ARG;
  MLM_REQUIRE(m->ctx, out && layer >= 0 && layer < m->cfg.n_layers, MLM_ERR_ARG,
              "mlm_llama_layer_tensors: layer %d of %d", layer, m->cfg.n_layers);
  const LayerBuf &L = m->layers[layer];
  const size_t rb = q4k_row_bytes(m->cfg.dim);
  out->attn_norm = L.attn_norm;
  out->ffn_norm = L.ffn_norm;
  out->wq = L.qkv;
  out->wk = L.qkv + (size_t)m->qdim() * rb;
  out->wv = L.v_type == MLM_TYPE_Q6_K ? L.wv6 : L.qkv + (size_t)(m->qdim() + m->kvdim()) * rb;
  out->wv_type = L.v_type;
  out->w_down_type = L.down_type;
  out->wo = L.wo;
  out->w_gate = L.gu;
  out->w_up = L.gu + (size_t)m->ffn() * rb;
  out->w_down = L.down;
  out->k_cache = L.kc;
  out->v_cache = L.vc;
  return MLM_OK;
}

extern "C" int mlm_llama_global_tensors(mlm_llama *m, mlm_llama_globals *out) {
  if (!m) return MLM_ERR_ARG;
  MLM_REQUIRE(m->ctx, out, MLM_ERR_ARG, "mlm_llama_global_tensors: null output");
  out->tok_embd = m->tok_embd;
  out->output_norm = m->out_norm;
  out->output = m->output;
  out->output_type = m->output_type;
  out->rope_freqs = m->rope_freqs;
  return MLM_OK;
}

extern "C" int mlm_llama_reset(mlm_llama *m) {
  if (!m) return MLM_ERR_ARG;
  m->pos = 0;
  std::fill(m->seq_pos.begin(), m->seq_pos.end(), 0);
  return MLM_OK;
}

extern "C" int mlm_llama_seq_position(const mlm_llama *m, int seq) {
  if (!m || seq < 0 || seq >= m->batch) return -1;
  return m->position(seq);
}

extern "C" int mlm_llama_set_position(mlm_llama *m, int pos) {
  if (!m) return MLM_ERR_ARG;
  MLM_REQUIRE(m->ctx, pos >= 0 && pos <= m->cfg.max_seq, MLM_ERR_ARG,
              "mlm_llama_set_position: %d outside [0, %d]", pos, m->cfg.max_seq);
  m->pos = pos;
  return MLM_OK;
}

extern "C" int mlm_llama_position(const mlm_llama *m) { return m ? m->pos : -1; }

extern "C" int mlm_llama_forward_layer(mlm_llama *m, int layer, float *hidden) {
  if (!m) return MLM_ERR_ARG;
  MLM_REQUIRE(m->ctx, hidden && layer >= 0 && layer < m->cfg.n_layers, MLM_ERR_ARG,
              "mlm_llama_forward_layer: layer %d of %d", layer, m->cfg.n_layers);
  MLM_REQUIRE(m->ctx, m->pos < m->cfg.max_seq, MLM_ERR_STATE,
              "mlm_llama_forward_layer: KV cache full (pos=%d, max=%d)", m->pos, m->cfg.max_seq);
  int st = m->set_state(0, m->pos, 0);
  if (st != MLM_OK) return st;
  return m->layer(layer, hidden);
}

extern "C" int mlm_llama_forward(mlm_llama *m, int token, float *logits) {
  if (!m) return MLM_ERR_ARG;
  MLM_REQUIRE(m->ctx, m->pos < m->cfg.max_seq, MLM_ERR_STATE,
              "mlm_llama_forward: KV cache full (pos=%d, max=%d)", m->pos, m->cfg.max_seq);
  MLM_REQUIRE(m->ctx, token >= 0 && token < m->cfg.vocab, MLM_ERR_ARG,
              "mlm_llama_forward: invalid token id %d (vocab %d)", token, m->cfg.vocab);
  int st = m->set_state(token, m->pos, 0);
  if (st == MLM_OK) st = m->step(true, logits);
  if (st == MLM_OK) m->pos += 1;
  return st;
}

extern "C" int mlm_llama_prefill(mlm_llama *m, const int32_t *tokens, int n, float *logits,
                                 int32_t *next) {
  if (!m) return MLM_ERR_ARG;
  mlm_ctx *ctx = m->ctx;
  MLM_REQUIRE(ctx, tokens && n > 0, MLM_ERR_ARG, "mlm_llama_prefill: no tokens");
  MLM_REQUIRE(ctx, m->pos + n <= m->cfg.max_seq, MLM_ERR_STATE,
              "mlm_llama_prefill: %d tokens at position %d exceed the cache (%d)", n, m->pos,
              m->cfg.max_seq);
  for (int i = 0; i < n; ++i)
    MLM_REQUIRE(ctx, tokens[i] >= 0 && tokens[i] < m->cfg.vocab, MLM_ERR_ARG,
                "mlm_llama_prefill: invalid token id %d at %d", tokens[i], i);
  int T = 0;
  for (int c0 = 0; c0 < n; c0 += T) {
    T = std::min(m->pf_chunk, n - c0);
    MLM_CUDA_TRY(ctx, cudaMemcpyAsync(m->pf_tokens, tokens + c0, sizeof(int32_t) * T,
                                      cudaMemcpyHostToDevice, ctx->stream));
    int st = m->prefill_chunk(T);
    if (st != MLM_OK) return st;
    m->pos += T;
  }
  // the output head on the last token, as a decode step ends
  const float *last = m->pf_hidden + (size_t)(T - 1) * m->cfg.dim;
  int st = m->head(last, logits);
  if (st != MLM_OK) return st;
  if (next)
    MLM_CUDA_TRY(ctx, cudaMemcpyAsync(next, m->state + kToken, sizeof(int32_t),
                                      cudaMemcpyDeviceToDevice, ctx->stream));
  return MLM_OK;
}

extern "C" int mlm_llama_decode_greedy(mlm_llama *m, int token, int steps, int32_t *tokens_out) {
  if (!m) return MLM_ERR_ARG;
  mlm_ctx *ctx = m->ctx;
  MLM_REQUIRE(ctx, tokens_out && steps > 0, MLM_ERR_ARG, "mlm_llama_decode_greedy: no output");
  MLM_REQUIRE(ctx, token >= 0 && token < m->cfg.vocab, MLM_ERR_ARG,
              "mlm_llama_decode_greedy: invalid token id %d", token);
  MLM_REQUIRE(ctx, m->pos + steps <= m->cfg.max_seq, MLM_ERR_STATE,
              "mlm_llama_decode_greedy: %d steps at position %d exceed the cache (%d)", steps,
              m->pos, m->cfg.max_seq);
  if (!m->step_exec) {
    // capture one step: embedding .. argmax, then record the token and move on
    MLM_CUDA_TRY(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    int st = m->step(true, nullptr);
    if (st == MLM_OK) {
      st = check_launch_pdl(ctx,
                            launch_pdl(advance_kernel, dim3(1), dim3(1), 0, ctx->stream,
                                       m->state, m->gen_tokens),
                            "mlm_llama_decode_greedy (advance)");
    }
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
    if (st != MLM_OK || e != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
      return st != MLM_OK ? st
                          : set_error(ctx, MLM_ERR_CUDA, "mlm_llama_decode_greedy: capture: %s",
                                      cudaGetErrorString(e));
    }
    m->step_graph = g;
    MLM_CUDA_TRY(ctx, cudaGraphInstantiate(&m->step_exec, g, 0));
  }
  int st = m->set_state(token, m->pos, 0);
  if (st != MLM_OK) return st;
  for (int i = 0; i < steps; ++i) MLM_CUDA_TRY(ctx, cudaGraphLaunch(m->step_exec, ctx->stream));
  MLM_CUDA_TRY(ctx, cudaMemcpyAsync(tokens_out, m->gen_tokens, sizeof(int32_t) * steps,
                                    cudaMemcpyDeviceToDevice, ctx->stream));
  m->pos += steps;
  return MLM_OK;
}

extern "C" int mlm_llama_prefill_seq(mlm_llama *m, int seq, const int32_t *tokens, int n,
                                     float *logits, int32_t *next) {
  if (!m) return MLM_ERR_ARG;
  MLM_REQUIRE(m->ctx, seq >= 0 && seq < m->batch, MLM_ERR_ARG,
              "mlm_llama_prefill_seq: sequence %d of %d", seq, m->batch);
  if (seq == 0) return mlm_llama_prefill(m, tokens, n, logits, next);
  const int saved = m->pos;
  m->pos = m->seq_pos[seq];
  m->cur = seq;
  const int st = mlm_llama_prefill(m, tokens, n, logits, next);
  m->seq_pos[seq] = m->pos;
  m->pos = saved;
  m->cur = 0;
  return st;
}

// device tokens and positions of the batch from the host
static int batch_begin(mlm_llama *m, const int32_t *tokens, int steps, const char *what) {
  mlm_ctx *ctx = m->ctx;
  MLM_REQUIRE(ctx, tokens, MLM_ERR_ARG, "%s: no tokens", what);
  std::vector<int> pos(m->batch);
  for (int b = 0; b < m->batch; ++b) {
    MLM_REQUIRE(ctx, tokens[b] >= 0 && tokens[b] < m->cfg.vocab, MLM_ERR_ARG,
                "%s: invalid token id %d for sequence %d", what, tokens[b], b);
    pos[b] = m->position(b);
    MLM_REQUIRE(ctx, pos[b] + steps <= m->cfg.max_seq, MLM_ERR_STATE,
                "%s: %d steps at position %d of sequence %d exceed the cache (%d)", what, steps,
                pos[b], b, m->cfg.max_seq);
  }
  MLM_CUDA_TRY(ctx, cudaMemcpyAsync(m->tok_b, tokens, sizeof(int32_t) * m->batch,
                                    cudaMemcpyHostToDevice, ctx->stream));
  MLM_CUDA_TRY(ctx, cudaMemcpyAsync(m->pos_b, pos.data(), sizeof(int) * m->batch,
                                    cudaMemcpyHostToDevice, ctx->stream));
  // the copies read pageable host memory: let them finish before `pos` goes
  MLM_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  return MLM_OK;
}

static void batch_advance(mlm_llama *m, int steps) {
  m->pos += steps;
  for (int b = 1; b < m->batch; ++b) m->seq_pos[b] += steps;
}

extern "C" int mlm_llama_forward_batch(mlm_llama *m, const int32_t *tokens, float *logits) {
  if (!m) return MLM_ERR_ARG;
  int st = batch_begin(m, tokens, 1, "mlm_llama_forward_batch");
  if (st == MLM_OK) st = m->step_batch(logits);
  if (st == MLM_OK) batch_advance(m, 1);
  return st;
}

extern "C" int mlm_llama_decode_greedy_batch(mlm_llama *m, const int32_t *tokens, int steps,
                                             int32_t *tokens_out) {
  if (!m) return MLM_ERR_ARG;
  mlm_ctx *ctx = m->ctx;
  MLM_REQUIRE(ctx, tokens_out && steps > 0, MLM_ERR_ARG, "mlm_llama_decode_greedy_batch: no output");
  int st = batch_begin(m, tokens, steps, "mlm_llama_decode_greedy_batch");
  if (st != MLM_OK) return st;
  if (!m->bstep_exec) {
    // capture one batched step: embedding .. argmax, then record the tokens
    MLM_CUDA_TRY(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    st = m->step_batch(nullptr);
    if (st == MLM_OK) {
      st = check_launch_pdl(ctx,
                            launch_pdl(advance_batch_kernel, dim3(1), dim3(64), 0, ctx->stream,
                                       m->state, m->pos_b, m->tok_b, m->gen_b, m->batch),
                            "mlm_llama_decode_greedy_batch (advance)");
    }
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
    if (st != MLM_OK || e != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
      return st != MLM_OK ? st
                          : set_error(ctx, MLM_ERR_CUDA, "mlm_llama_decode_greedy_batch: capture: %s",
                                      cudaGetErrorString(e));
    }
    m->bstep_graph = g;
    MLM_CUDA_TRY(ctx, cudaGraphInstantiate(&m->bstep_exec, g, 0));
  }
  if ((st = m->set_state(0, 0, 0)) != MLM_OK) return st;
  for (int i = 0; i < steps; ++i) MLM_CUDA_TRY(ctx, cudaGraphLaunch(m->bstep_exec, ctx->stream));
  MLM_CUDA_TRY(ctx, cudaMemcpyAsync(tokens_out, m->gen_b, sizeof(int32_t) * steps * m->batch,
                                    cudaMemcpyDeviceToDevice, ctx->stream));
  batch_advance(m, steps);
  return MLM_OK;
}
