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
// End of a step whose position lives on the device: record the token and advance.
__global__ void decoder_advance_kernel(int* pos, const int* token, int* history, int max_t) {
  pyre::pdl_wait();
  pyre::pdl_trigger();
  const int p = *pos;
  if (p >= 0 && p < max_t) {
    history[p + 1] = *token;
    *pos = p + 1;
  }
}
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
  const int H = d->H, qw = d->nq * d->hd, kw = d->nkv * d->hd, nqkv = qw + 2 * kw;
  int rc = pyre_embed_rms_norm(token_in, 1, d->embedding, d->V, H, d->layers[0].ln1, d->eps, d->x, d->xn, d->status,
                               stream);
  if (rc) return rc;
  for (int i = 0; i < d->n_layers; ++i) {
    const pyre_decoder_layer& L = d->layers[i];
    rc = pyre_q80_linear_bias(d->xn, PYRE_F32, 1, H, L.qkv_w, d->scale_dtype, nqkv, L.qkv_bias, d->qkv, L.qkv_ws,
                              L.qkv_ws_bytes, stream);
    if (rc) return rc;
    rc = d->pos_dev == nullptr
             ? pyre_attn_decode_step(d->qkv, d->qkv + qw, d->qkv + qw + kw, pos, L.rope, d->rope_fraction, d->nq,
                                     d->nkv, d->hd, L.k_cache, L.v_cache, d->max_t, mask_lo, mask_hi, d->attn,
                                     L.attn_ws, L.attn_ws_bytes, stream)
             : pyre_attn_decode_step_dev(d->qkv, d->qkv + qw, d->qkv + qw + kw, d->pos_dev, pos, L.rope,
                                         d->rope_fraction, d->nq, d->nkv, d->hd, L.k_cache, L.v_cache, d->max_t,
                                         mask_lo, mask_hi, d->attn, L.attn_ws, L.attn_ws_bytes, stream);
    if (rc) return rc;
    // O projection of this rank's heads; with tensor parallelism the ranks' partials are summed
    // in the epilogue (the head-partitioned root concatenates the heads' outputs before Wo,
    // root_node.py:851-858: the sum over head groups of attn_g @ Wo[rows of g] is that product)
    rc = d->comm == nullptr
             ? pyre_q80_linear(d->attn, PYRE_F32, 1, qw, L.o_w, d->scale_dtype, H, d->ao, L.o_ws, L.o_ws_bytes, stream)
             : pyre_ffn_down_q80(d->attn, PYRE_F32, 1, qw, L.o_w, d->scale_dtype, H, d->ao, L.o_ws, L.o_ws_bytes,
                                 d->comm, stream);
    if (rc) return rc;
    rc = pyre_add_rms_norm(d->x, d->ao, 1, H, L.ln2, d->eps, d->x, d->hn, stream);
    if (rc) return rc;
    rc = pyre_ffn_decode_q80(d->hn, PYRE_F32, 1, H, L.gateup_w, L.gated, L.down_w, d->scale_dtype, d->ffn_width, d->f,
                             L.ffn_ws, L.ffn_ws_bytes, d->comm, stream);
    if (rc) return rc;
    const bool last = i + 1 == d->n_layers;
    rc = pyre_add_rms_norm(d->x, d->f, 1, H, last ? nullptr : d->layers[i + 1].ln1, d->eps, d->x,
                           last ? nullptr : d->xn, stream);
    if (rc) return rc;
  }
  const int lm_V = d->lm_V > 0 ? d->lm_V : d->V;
  rc = pyre_lm_head_argmax(d->x, 1, H, d->final_norm, d->eps, d->lm_head, lm_V, d->lm_v0, logits, token_out, d->key,
                           d->lm_ws, d->lm_ws_bytes, stream);
  if (rc) return rc;
  if (d->comm != nullptr) {
    // vocabulary split over the ranks: the token is the best of the ranks' keys
    rc = pyre_argmax_combine(d->comm, d->key, 1, token_out, nullptr, stream);
    if (rc) return rc;
  }
  if (d->pos_dev == nullptr) return rc;
  PYRE_CHECK_ARG(d->history != nullptr, "pyre_decoder_step: pos_dev needs a history buffer");
  PYRE_CUDA_TRY(pyre::launch_pdl(decoder_advance_kernel, dim3(1), dim3(1), 0, static_cast<cudaStream_t>(stream),
                                 d->pos_dev, static_cast<const int*>(token_out), d->history, d->max_t));
  return PYRE_OK;
}

extern "C" int pyre_decoder_struct_sizes(int64_t* layer_bytes, int64_t* desc_bytes) {
  PYRE_CHECK_ARG(layer_bytes != nullptr && desc_bytes != nullptr, "pyre_decoder_struct_sizes: null pointer");
  *layer_bytes = static_cast<int64_t>(sizeof(pyre_decoder_layer));
  *desc_bytes = static_cast<int64_t>(sizeof(pyre_decoder_desc));
  return PYRE_OK;
}
