// Host-side decode step of a Llama-style decoder: the launch sequence of one greedy token
// in one C call, so a step costs ~6 launches per layer of host time instead of a Python
// round trip per launch.
//
// One step (src/orchestrator/generator.py:117-131 over root_node.py:739-1007):
//   embed_rms_norm                  x = f32(table[token]), xn = rms_norm(x, ln1[0])
//   per layer:
//     q80 linear                    qkv = xn @ [Wq | Wk | Wv]
//     attention decode step         RoPE at `pos`, clip, KV append, flash-decoding, mask
//     q80 linear                    ao = attn @ Wo
//     add_rms_norm                  x += ao, hn = rms_norm(x, ln2)
//     FFN decode                    f = down(silu(hn @ Wgate) * (hn @ Wup))
//     add_rms_norm                  x += f, xn = rms_norm(x, ln1[next])   (add only after the last)
//   lm_head argmax                  final RMSNorm, logits, greedy token
// Every buffer is the caller's (device memory it allocated once); nothing is allocated here.
// With desc->pos_dev the position is read on the device and advanced by the step itself, so
// one captured step replays for consecutive positions.
#include "comm.cuh"

namespace {
// End of a step whose position lives on the device: record the B tokens (history [B, max_t + 1])
// and advance the position.
__global__ void decoder_advance_kernel(int* pos, const int* token, int* history, int max_t, int B) {
  pyre::pdl_wait();
  pyre::pdl_trigger();
  const int p = *pos;
  if (p >= 0 && p < max_t) {
    for (int b = 0; b < B; ++b) history[static_cast<int64_t>(b) * (max_t + 1) + p + 1] = token[b];
    *pos = p + 1;
  }
}

constexpr int kRowGroup = PYRE_FUSED_REDUCE_MAX_T;   // tokens per projection / FFN call
}  // namespace

extern "C" int pyre_decoder_step(const pyre_decoder_desc* d, const int* token_in, int pos, int mask_lo, int mask_hi,
                                 int* token_out, float* logits, void* stream) {
  PYRE_CHECK_ARG(d != nullptr && d->layers != nullptr && token_in != nullptr && token_out != nullptr,
                 "pyre_decoder_step: null pointer");
  PYRE_CHECK_ARG(d->n_layers >= 1 && d->H >= 1 && d->nq >= 1 && d->nkv >= 1 && d->hd >= 1 && d->ffn_width >= 1 &&
                     d->V >= 1,
                 "pyre_decoder_step: bad sizes");
  PYRE_CHECK_ARG(pos >= 0 && pos < d->max_t, "pyre_decoder_step: position outside the KV cache");
  PYRE_CHECK_ARG(d->lm_V >= 0 && d->lm_v0 >= 0 && d->lm_v0 + (d->lm_V > 0 ? d->lm_V : d->V) <= d->V,
                 "pyre_decoder_step: lm_head rows outside the vocabulary");
  PYRE_CHECK_ARG(d->comm == nullptr || d->comm->hidden == d->H,
                 "pyre_decoder_step: the communicator's hidden size differs from H");
  const int B = d->batch > 1 ? d->batch : 1;
  PYRE_CHECK_ARG(B <= 64, "pyre_decoder_step: at most 64 sequences");
  PYRE_CHECK_ARG(B == 1 || (mask_lo == 0 && mask_hi == 0), "pyre_decoder_step: a batch takes no prefill mask");
  const int H = d->H, qw = d->nq * d->hd, kw = d->nkv * d->hd, nqkv = qw + 2 * kw;
  const int lm_V = d->lm_V > 0 ? d->lm_V : d->V;
  int rc = pyre_embed_rms_norm(token_in, B, d->embedding, d->V, H, d->layers[0].ln1, d->eps, d->x, d->xn, d->status,
                               stream);
  if (rc) return rc;
  for (int i = 0; i < d->n_layers; ++i) {
    const pyre_decoder_layer& L = d->layers[i];
    for (int r0 = 0; r0 < B; r0 += kRowGroup) {
      const int n = B - r0 < kRowGroup ? B - r0 : kRowGroup;
      rc = pyre_q80_linear_bias(d->xn + static_cast<int64_t>(r0) * H, PYRE_F32, n, H, L.qkv_w, d->scale_dtype, nqkv,
                                L.qkv_bias, d->qkv + static_cast<int64_t>(r0) * nqkv, L.qkv_ws, L.qkv_ws_bytes, stream);
      if (rc) return rc;
    }
    if (B > 1)
      rc = pyre_attn_decode_step_batch(d->qkv, d->qkv + qw, d->qkv + qw + kw, nqkv, B, d->pos_dev, pos, L.rope,
                                       d->rope_fraction, d->nq, d->nkv, d->hd, L.k_cache, L.v_cache, d->max_t, d->attn,
                                       L.attn_ws, L.attn_ws_bytes, stream);
    else if (d->pos_dev == nullptr)
      rc = pyre_attn_decode_step(d->qkv, d->qkv + qw, d->qkv + qw + kw, pos, L.rope, d->rope_fraction, d->nq, d->nkv,
                                 d->hd, L.k_cache, L.v_cache, d->max_t, mask_lo, mask_hi, d->attn, L.attn_ws,
                                 L.attn_ws_bytes, stream);
    else
      rc = pyre_attn_decode_step_dev(d->qkv, d->qkv + qw, d->qkv + qw + kw, d->pos_dev, pos, L.rope, d->rope_fraction,
                                     d->nq, d->nkv, d->hd, L.k_cache, L.v_cache, d->max_t, mask_lo, mask_hi, d->attn,
                                     L.attn_ws, L.attn_ws_bytes, stream);
    if (rc) return rc;
    for (int r0 = 0; r0 < B; r0 += kRowGroup) {
      const int n = B - r0 < kRowGroup ? B - r0 : kRowGroup;
      const float* a = d->attn + static_cast<int64_t>(r0) * qw;
      float* ao = d->ao + static_cast<int64_t>(r0) * H;
      // O projection of this rank's heads; with tensor parallelism the ranks' partials are
      // summed in the epilogue (the head-partitioned root concatenates the heads' outputs
      // before Wo, root_node.py:851-858: the sum over head groups of attn_g @ Wo[rows of g] is
      // that product)
      rc = d->comm == nullptr
               ? pyre_q80_linear(a, PYRE_F32, n, qw, L.o_w, d->scale_dtype, H, ao, L.o_ws, L.o_ws_bytes, stream)
               : pyre_ffn_down_q80(a, PYRE_F32, n, qw, L.o_w, d->scale_dtype, H, ao, L.o_ws, L.o_ws_bytes, d->comm,
                                   stream);
      if (rc) return rc;
    }
    rc = pyre_add_rms_norm(d->x, d->ao, B, H, L.ln2, d->eps, d->x, d->hn, stream);
    if (rc) return rc;
    for (int r0 = 0; r0 < B; r0 += kRowGroup) {
      const int n = B - r0 < kRowGroup ? B - r0 : kRowGroup;
      rc = pyre_ffn_decode_q80(d->hn + static_cast<int64_t>(r0) * H, PYRE_F32, n, H, L.gateup_w, L.gated, L.down_w,
                               d->scale_dtype, d->ffn_width, d->f + static_cast<int64_t>(r0) * H, L.ffn_ws,
                               L.ffn_ws_bytes, d->comm, stream);
      if (rc) return rc;
    }
    const bool last = i + 1 == d->n_layers;
    rc = pyre_add_rms_norm(d->x, d->f, B, H, last ? nullptr : d->layers[i + 1].ln1, d->eps, d->x,
                           last ? nullptr : d->xn, stream);
    if (rc) return rc;
  }
  for (int r0 = 0; r0 < B; r0 += kRowGroup) {
    const int n = B - r0 < kRowGroup ? B - r0 : kRowGroup;
    rc = pyre_lm_head_argmax(d->x + static_cast<int64_t>(r0) * H, n, H, d->final_norm, d->eps, d->lm_head, lm_V,
                             d->lm_v0, logits != nullptr ? logits + static_cast<int64_t>(r0) * lm_V : nullptr,
                             token_out + r0, d->key + r0, d->lm_ws, d->lm_ws_bytes, stream);
    if (rc) return rc;
    if (d->comm != nullptr) {
      // vocabulary split over the ranks: the token is the best of the ranks' keys
      rc = pyre_argmax_combine(d->comm, d->key + r0, n, token_out + r0, nullptr, stream);
      if (rc) return rc;
    }
  }
  if (d->pos_dev == nullptr) return rc;
  PYRE_CHECK_ARG(d->history != nullptr, "pyre_decoder_step: pos_dev needs a history buffer");
  PYRE_CUDA_TRY(pyre::launch_pdl(decoder_advance_kernel, dim3(1), dim3(1), 0, static_cast<cudaStream_t>(stream),
                                 d->pos_dev, static_cast<const int*>(token_out), d->history, d->max_t, B));
  return PYRE_OK;
}

extern "C" int pyre_decoder_struct_sizes(int64_t* layer_bytes, int64_t* desc_bytes) {
  PYRE_CHECK_ARG(layer_bytes != nullptr && desc_bytes != nullptr, "pyre_decoder_struct_sizes: null pointer");
  *layer_bytes = static_cast<int64_t>(sizeof(pyre_decoder_layer));
  *desc_bytes = static_cast<int64_t>(sizeof(pyre_decoder_desc));
  return PYRE_OK;
}
