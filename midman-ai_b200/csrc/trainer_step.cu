// The training step on the device: forward (model.rs:127-165), cross-entropy
// (ops_reduce.rs:236-276), backward (the reference's autograd replayed as fused
// kernels), data-parallel gradient averaging, clip and AdamW.
//
// Parameters keep the reference's layout ([in, out] row-major linears), so each
// linear's three products map onto the GEMM's operand majors as
//   Y  = X W      -> A = X K-major,  B = W MN-major
//   dX = dY W^T   -> A = dY K-major, B = W K-major
//   dW = X^T dY   -> A = X MN-major, B = dY MN-major
// and no transposed copies are made (the reference copies W for the tied head,
// model.rs:163, and B for every gemm_nt, kernels.rs:66-75).
#include "nccl_api.h"

#include <cmath>
#include <cstring>
#include <stdexcept>

#include "attention.h"
#include "device.h"
#include "trainer.h"

namespace mm {

namespace {
void nccl_ok(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw std::runtime_error(std::string(what) + ": " + nccl().GetErrorString(r));
}
}  // namespace

void Trainer::forward(int B, int T, bool train) {
  const int N = B * T;
  const int D = static_cast<int>(cfg_.d_model), F = static_cast<int>(cfg_.d_ff), KV = static_cast<int>(cfg_.kv_dim());
  const int V = static_cast<int>(cfg_.vocab), H = static_cast<int>(cfg_.n_heads), Hkv = static_cast<int>(cfg_.n_kv_heads);
  const int hd = static_cast<int>(cfg_.head_dim());
  const float eps = cfg_.norm_eps;
  const AttnShape shape{B, T, H, Hkv, hd, D, KV, KV, D, 1.0f / std::sqrt(static_cast<float>(hd))};
  const int L = static_cast<int>(cfg_.n_layers);
  // The k/v projections (and RoPE of k) and the up projection run on the side
  // stream beside q and gate, which read the same normalized input; the main
  // stream waits for them before attention and SwiGLU. One stream with
  // profiling on and in 3xTF32 (its split operands share one scratch arena).
  const bool dual = side_stream_ != nullptr && !profiling_ && precision_ == kPrecisionTF32;
  cudaStream_t ws = dual ? side_stream_ : stream_;
  auto to_side = [&] {
    if (!dual) return;
    check_cuda(cudaEventRecord(side_ev_[0], stream_), "event");
    check_cuda(cudaStreamWaitEvent(ws, side_ev_[0], 0), "wait");
  };
  auto from_side = [&] {
    if (!dual) return;
    check_cuda(cudaEventRecord(side_ev_[1], ws), "event");
    check_cuda(cudaStreamWaitEvent(stream_, side_ev_[1], 0), "wait");
  };
  // under optimizer sharding, each bucket's parameters may still be arriving from their owner
  wait_params(0);
  embedding_forward(d_ids_, N, P_ + layout_.embed, static_cast<int>(cfg_.vocab), D, acts_[0].x,
                    device_context().d_err, stream_);
  launches_ += 1;
  for (int l = 0; l < L; ++l) {
    Layer& a = acts_[l];
    const BlockOffsets& bo = layout_.blocks[l];
    wait_params(1 + l);
    float* next_x = (l + 1 < L) ? acts_[l + 1].x : x_final_;
    // h = x + attention(attn_norm(x)) (block.rs:78-79)
    rmsnorm_forward(a.x, P_ + bo.attn_norm, N, D, eps, a.xn1, a.rstd1, stream_);
    to_side();
    gemm(N, KV, D, a.xn1, D, false, P_ + bo.k, KV, true, a.k, KV, nullptr, 0, ws);
    gemm(N, KV, D, a.xn1, D, false, P_ + bo.v, KV, true, a.v, KV, nullptr, 0, ws, true);  // xn1 again
    rope(a.k, N, T, Hkv, hd, KV, d_cos_, d_sin_, false, ws);
    gemm(N, D, D, a.xn1, D, false, P_ + bo.q, D, true, a.q, D, nullptr, 0, nullptr, true);
    rope(a.q, N, T, H, hd, D, d_cos_, d_sin_, false, stream_);
    from_side();
    const double attn_flops = 2.0 * B * H * static_cast<double>(T) * (T + 1) * hd;  // QK^T and PV, causal half
    int slot = prof_begin();
    if (attn_tc_)  // fused: the scores stay on chip
      attention_forward_flash(shape, a.q, a.k, a.v, a.o, a.lse, device_context().d_err, stream_);
    else if (attn_3x_)
      attention_forward_3x(shape, a.q, a.k, a.v, a.o, a.lse, attn3_ws_, device_context().d_err, stream_);
    else
      attention_forward(shape, a.q, a.k, a.v, a.o, a.lse, stream_);
    prof_end(slot, "attention_fwd", attn_flops);
    gemm(N, D, D, a.o, D, false, P_ + bo.o, D, true, a.h, D, a.x, D);
    // out = h + swiglu(mlp_norm(h)) (mlp.rs:20-24)
    rmsnorm_forward(a.h, P_ + bo.mlp_norm, N, D, eps, a.xn2, a.rstd2, stream_);
    to_side();
    gemm(N, F, D, a.xn2, D, false, P_ + bo.up, F, true, a.u, F, nullptr, 0, ws);
    gemm(N, F, D, a.xn2, D, false, P_ + bo.gate, F, true, a.g, F, nullptr, 0, nullptr, true);  // xn2 again
    from_side();
    swiglu_forward(a.g, a.u, a.act, static_cast<long long>(N) * F, stream_);
    gemm(N, D, F, a.act, F, false, P_ + bo.down, D, true, next_x, D, a.h, D);
    launches_ += 6;  // two RMSNorms, two RoPEs, attention, SwiGLU (GEMMs are counted in gemm())
  }
  wait_params(L + 1);
  rmsnorm_forward(x_final_, P_ + layout_.final_norm, N, D, eps, xf_, rstdf_, stream_);
  launches_ += 1;
  if (cfg_.tie)  // logits = xf E^T: E [V, D] is already K-major for this product
    gemm(N, V, D, xf_, D, false, P_ + layout_.embed, D, false, logits_, V, nullptr, 0);
  else
    gemm(N, V, D, xf_, D, false, P_ + layout_.lm_head, V, true, logits_, V, nullptr, 0);
  (void)train;
}

void Trainer::backward(int B, int T) {
  const int N = B * T;
  const int D = static_cast<int>(cfg_.d_model), F = static_cast<int>(cfg_.d_ff), KV = static_cast<int>(cfg_.kv_dim());
  const int V = static_cast<int>(cfg_.vocab), H = static_cast<int>(cfg_.n_heads), Hkv = static_cast<int>(cfg_.n_kv_heads);
  const int hd = static_cast<int>(cfg_.head_dim());
  const AttnShape shape{B, T, H, Hkv, hd, D, KV, KV, D, 1.0f / std::sqrt(static_cast<float>(hd))};
  const int L = static_cast<int>(cfg_.n_layers);
  // The weight-gradient products are off the path the gradient flows down: they
  // run on the side stream (ws), each after an event of the main stream that
  // made its inputs, while the main stream goes on; the main stream waits for
  // them before it overwrites a buffer they read (the scratch dh, dq, dk, dv, dx)
  // and before the gradients are used. One stream with profiling on (per-kernel
  // times) and in 3xTF32 (its split operands share one scratch arena).
  const bool dual = side_stream_ != nullptr && !profiling_ && precision_ == kPrecisionTF32;
  cudaStream_t ws = dual ? side_stream_ : stream_;
  auto to_side = [&] {  // the side stream waits for the main stream's work so far
    if (!dual) return;
    check_cuda(cudaEventRecord(side_ev_[0], stream_), "event");
    check_cuda(cudaStreamWaitEvent(ws, side_ev_[0], 0), "wait");
  };
  auto side_mark = [&](int e) {  // an event after the side stream's work so far
    if (dual) check_cuda(cudaEventRecord(side_ev_[e], ws), "event");
  };
  auto main_waits = [&](int e) {
    if (dual) check_cuda(cudaStreamWaitEvent(stream_, side_ev_[e], 0), "wait");
  };
  // logits_ holds d loss / d logits. Head products first (the tape starts there):
  if (cfg_.tie) {
    gemm(N, D, V, logits_, V, false, P_ + layout_.embed, D, true, tmp_, D, nullptr, 0);
    to_side();
    gemm(V, D, N, logits_, V, true, xf_, D, true, G_ + layout_.embed, D, nullptr, 0, ws);
  } else {
    gemm(N, D, V, logits_, V, false, P_ + layout_.lm_head, V, false, tmp_, D, nullptr, 0);
    to_side();
    gemm(D, V, N, xf_, D, true, logits_, V, true, G_ + layout_.lm_head, V, nullptr, 0, ws);
    check_cuda(cudaMemsetAsync(G_ + layout_.embed, 0, static_cast<size_t>(V) * D * 4, ws), "zero dE");
  }
  side_mark(3);  // the head's share of dE
  const int c = 0;  // dx_[c] carries the gradient down the residual stream
  float* dx = dx_[c];
  float* dh = dx_[1 - c];
  rmsnorm_backward(x_final_, P_ + layout_.final_norm, rstdf_, tmp_, N, D, dx, nullptr, G_ + layout_.final_norm,
                   norm_ws_, stream_);
  launches_ += 2;
  for (int l = L - 1; l >= 0; --l) {
    Layer& a = acts_[l];
    const BlockOffsets& bo = layout_.blocks[l];
    // x_next = h + act Wd
    to_side();  // dx of this layer is ready
    gemm(F, D, N, a.act, F, true, dx, D, true, G_ + bo.down, D, nullptr, 0, ws);
    side_mark(1);  // dx read
    gemm(N, F, D, dx, D, false, P_ + bo.down, D, false, dact_, F, nullptr, 0, nullptr, true);  // dx again
    swiglu_backward(a.g, a.u, dact_, static_cast<long long>(N) * F, stream_);  // g <- dg, u <- du
    to_side();
    gemm(D, F, N, a.xn2, D, true, a.g, F, true, G_ + bo.gate, F, nullptr, 0, ws);
    gemm(D, F, N, a.xn2, D, true, a.u, F, true, G_ + bo.up, F, nullptr, 0, ws, true);
    {  // dxn = dg Wg^T + du Wu^T, one accumulator
      const GemmSegment segs[2] = {{{a.g, F, false}, {P_ + bo.gate, F, false}, F},
                                   {{a.u, F, false}, {P_ + bo.up, F, false}, F}};
      gemm_sum(N, D, segs, 2, dxn_, D, nullptr, 0, nullptr, true);  // dg, du again
    }
    if (l + 1 < L) main_waits(2);  // the layer above's products have read dh, dq, dk, dv
    rmsnorm_backward(a.h, P_ + bo.mlp_norm, a.rstd2, dxn_, N, D, dh, dx, G_ + bo.mlp_norm, norm_ws_, stream_);
    // h = x + o Wo
    to_side();
    gemm(D, D, N, a.o, D, true, dh, D, true, G_ + bo.o, D, nullptr, 0, ws);
    gemm(N, D, D, dh, D, false, P_ + bo.o, D, false, do_, D, nullptr, 0, nullptr, true);  // dh again
    int slot = prof_begin();
    if (attn_tc_) {
      const BwdSide side{side_stream_, attn_side_ready_, attn_side_done_};
      attention_backward_flash(shape, a.q, a.k, a.v, a.o, a.lse, do_, D, dq_, dk_, dv_, delta_, device_context().d_err,
                               stream_, &side);
    } else if (attn_3x_) {
      attention_backward_3x(shape, a.q, a.k, a.v, a.o, a.lse, do_, D, dq_, dk_, dv_, attn3_ws_, device_context().d_err,
                            stream_);
    } else {
      attention_backward(shape, a.q, a.k, a.v, a.o, a.lse, do_, D, dq_, dk_, dv_, delta_, stream_);
    }
    // dV, dP, dQ, dK: four causal products (the recomputed scores are not counted)
    prof_end(slot, "attention_bwd", 4.0 * B * H * static_cast<double>(T) * (T + 1) * hd);
    rope(dq_, N, T, H, hd, D, d_cos_, d_sin_, true, stream_);
    rope(dk_, N, T, Hkv, hd, KV, d_cos_, d_sin_, true, stream_);
    to_side();
    gemm(D, D, N, a.xn1, D, true, dq_, D, true, G_ + bo.q, D, nullptr, 0, ws);
    gemm(D, KV, N, a.xn1, D, true, dk_, KV, true, G_ + bo.k, KV, nullptr, 0, ws, true);
    gemm(D, KV, N, a.xn1, D, true, dv_, KV, true, G_ + bo.v, KV, nullptr, 0, ws, true);
    side_mark(2);  // this layer's weight gradients are done
    {  // dxn = dq Wq^T + dk Wk^T + dv Wv^T, one accumulator
      const GemmSegment segs[3] = {{{dq_, D, false}, {P_ + bo.q, D, false}, D},
                                   {{dk_, KV, false}, {P_ + bo.k, KV, false}, KV},
                                   {{dv_, KV, false}, {P_ + bo.v, KV, false}, KV}};
      gemm_sum(N, D, segs, 3, dxn_, D, nullptr, 0, nullptr, true);  // dq, dk, dv again
    }
    main_waits(1);  // the down projection's product has read dx
    rmsnorm_backward(a.x, P_ + bo.attn_norm, a.rstd1, dxn_, N, D, dx, dh, G_ + bo.attn_norm, norm_ws_, stream_);
    launches_ += 10;  // SwiGLU, two RMSNorm backwards (2 kernels each), attention backward (3), two RoPEs
    if (world_ > 1) {
      // This layer's gradients are final: average them while the next layer's
      // backward runs (a bucket per layer, in reverse parameter order).
      check_cuda(cudaEventRecord(layer_done_[l], stream_), "event");
      check_cuda(cudaStreamWaitEvent(comm_stream_, layer_done_[l], 0), "wait");
      if (dual) check_cuda(cudaStreamWaitEvent(comm_stream_, side_ev_[2], 0), "wait");
      reduce_bucket(1 + l);
    }
  }
  main_waits(2);  // every weight gradient of the blocks
  main_waits(3);  // and the head's share of dE
  // the embedding's share, added after the head's (ops_shape.rs:262-272)
  embedding_backward(d_uniq_, d_off_, d_pos_, n_uniq_, dx, D, G_ + layout_.embed, stream_);
  launches_ += 1;
  if (world_ > 1) {
    check_cuda(cudaEventRecord(layer_done_[L], stream_), "event");
    check_cuda(cudaStreamWaitEvent(comm_stream_, layer_done_[L], 0), "wait");
    reduce_bucket(0);
    reduce_bucket(L + 1);
    nccl_ok(nccl().AllReduce(d_loss_, d_loss_, 1, ncclDouble, ncclAvg, static_cast<ncclComm_t>(comm_), comm_stream_),
            "ncclAllReduce(loss)");
    check_cuda(cudaEventRecord(comm_done_, comm_stream_), "event");
    check_cuda(cudaStreamWaitEvent(stream_, comm_done_, 0), "wait");
  }
}

StepOut Trainer::finish_step(float lr, const AdamHyper& h, bool update) {
  finish_launch(lr, h, update);
  return finish_collect(update);
}

void Trainer::finish_launch(float lr, const AdamHyper& h, bool update) {
  const long long total = static_cast<long long>(layout_.total);
  if (owner_reduce_) {
    // each rank sums the grid blocks of its own range (reduced there); the others'
    // blocks are 0, so the summed partials are the grid of the whole gradient
    sumsq_partials(G_, total, d_partials_, stream_, static_cast<long long>(shard_begin(rank_)),
                   static_cast<long long>(shard_end(rank_)));
    nccl_ok(nccl().AllReduce(d_partials_, d_partials_, kNormBlocks, ncclDouble, ncclSum,
                             static_cast<ncclComm_t>(comm_), stream_),
            "ncclAllReduce(norm partials)");
  } else {
    sumsq_partials(G_, total, d_partials_, stream_);
  }
  finish_norm(d_partials_, d_loss_, h.clip_norm, d_norm_, stream_);
  launches_ += 2;
  if (update) {
    // adamw.rs:192-196: bias corrections in f64 for the step about to be taken
    const double t = static_cast<double>(adam_steps_ + 1);
    const float bias1 = static_cast<float>(1.0 - std::pow(static_cast<double>(h.beta1), t));
    const float bias2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(static_cast<double>(h.beta2), t)));
    const float step_size = lr / bias1;
    if (!zero1_ && side_stream_ && !profiling_) {
      // Bucket by bucket on the side stream, each bucket's event the next
      // forward's wait (wait_params): the HBM-bound update of the later buckets
      // runs beside the tensor-bound forward of the first layers.
      check_cuda(cudaEventRecord(update_done_, stream_), "event");
      check_cuda(cudaStreamWaitEvent(side_stream_, update_done_, 0), "wait");
      for (size_t b = 0; b < bucket_chunks_.size(); ++b) {
        const int c0 = bucket_chunks_[b].first, n = bucket_chunks_[b].second - c0;
        adamw_step(d_chunks_ + c0, n, P_, G_, M_, V_, 0, d_norm_, lr, h.beta1, h.beta2, h.eps, h.weight_decay,
                   step_size, bias2_sqrt, side_stream_);
        check_cuda(cudaEventRecord(gathered_[b], side_stream_), "event");
        launches_ += n > 0 ? 1 : 0;
      }
      gather_pending_ = true;
    } else {
      adamw_step(d_chunks_, n_chunks_, P_, G_, M_, V_, static_cast<long long>(mv_begin()), d_norm_, lr, h.beta1,
                 h.beta2, h.eps, h.weight_decay, step_size, bias2_sqrt, stream_);
      launches_ += 1;
      if (zero1_ && world_ > 1) broadcast_params();
    }
  }
  check_cuda(cudaMemcpyAsync(h_out_, d_loss_, sizeof(double), cudaMemcpyDeviceToHost, stream_), "loss D2H");
  check_cuda(cudaMemcpyAsync(h_out_ + 2, d_norm_, 3 * sizeof(float), cudaMemcpyDeviceToHost, stream_), "norm D2H");
}

StepOut Trainer::finish_collect(bool update) {
  check_device("training step");  // synchronizes the stream
  if (profiling_) prof_collect();
  double loss;
  std::memcpy(&loss, h_out_, sizeof(double));
  StepOut out;
  out.loss = static_cast<float>(loss);
  out.grad_norm = h_out_[2];
  out.ok = h_out_[4] != 0.0f;
  if (update && out.ok) ++adam_steps_;
  return out;
}

void Trainer::stage_batch(const int32_t* inputs, const int32_t* targets) {
  upload_batch(inputs, targets, batch_, seq_);
}

StepOut Trainer::step_staged(float lr, const AdamHyper& h) {
  launch_step(lr, h);
  return collect_step();
}

void Trainer::launch_step(float lr, const AdamHyper& h) {
  if (!(std::isfinite(lr) && lr >= 0.0f)) throw std::invalid_argument("lr must be finite and not negative");
  const int N = batch_ * seq_;
  owner_reduce_ = zero1_ && world_ > 1;
  grads_partial_ = owner_reduce_;
  forward(batch_, seq_, true);
  cross_entropy(logits_, cfg_.vocab, d_tgt_, N, static_cast<int>(cfg_.vocab), 1.0f / static_cast<float>(N), row_loss_,
                device_context().d_err, stream_);
  mean_loss(row_loss_, N, d_loss_, stream_);
  launches_ += 2;
  backward(batch_, seq_);
  finish_launch(lr, h, true);
}

StepOut Trainer::collect_step() { return finish_collect(true); }

StepOut Trainer::train_step(const int32_t* inputs, const int32_t* targets, float lr, const AdamHyper& h) {
  stage_batch(inputs, targets);
  return step_staged(lr, h);
}

float Trainer::loss_and_grads(const int32_t* inputs, const int32_t* targets) {
  stage_batch(inputs, targets);
  owner_reduce_ = false;  // whole gradients on every rank
  grads_partial_ = false;
  const int N = batch_ * seq_;
  forward(batch_, seq_, true);
  cross_entropy(logits_, cfg_.vocab, d_tgt_, N, static_cast<int>(cfg_.vocab), 1.0f / static_cast<float>(N), row_loss_,
                device_context().d_err, stream_);
  mean_loss(row_loss_, N, d_loss_, stream_);
  backward(batch_, seq_);
  AdamHyper h;
  h.clip_norm = 1e30f;
  return finish_step(0.0f, h, false).loss;
}

float Trainer::eval(const int32_t* inputs, const int32_t* targets, int B, int T, int32_t* predictions) {
  upload_batch(inputs, targets, B, T);
  const int N = B * T;
  forward(B, T, false);
  if (predictions) {
    argmax_rows(logits_, cfg_.vocab, N, static_cast<int>(cfg_.vocab), d_pred_, stream_);
    check_cuda(cudaMemcpyAsync(predictions, d_pred_, N * 4, cudaMemcpyDeviceToHost, stream_), "predictions");
  }
  cross_entropy(logits_, cfg_.vocab, d_tgt_, N, static_cast<int>(cfg_.vocab), 1.0f / static_cast<float>(N), row_loss_,
                device_context().d_err, stream_);
  mean_loss(row_loss_, N, d_loss_, stream_);
  check_cuda(cudaMemcpyAsync(h_out_, d_loss_, sizeof(double), cudaMemcpyDeviceToHost, stream_), "loss D2H");
  check_device("eval");
  double loss;
  std::memcpy(&loss, h_out_, sizeof(double));
  return static_cast<float>(loss);
}

void Trainer::logits(const int32_t* inputs, int B, int T, float* host_out) {
  upload_batch(inputs, nullptr, B, T);
  forward(B, T, false);
  check_cuda(cudaMemcpyAsync(host_out, logits_, static_cast<size_t>(B) * T * cfg_.vocab * 4, cudaMemcpyDeviceToHost,
                             stream_),
             "logits D2H");
  check_device("logits");
}

void Trainer::attention_maps(const int32_t* inputs, int B, int T, float* host_out) {
  upload_batch(inputs, nullptr, B, T);
  forward(B, T, false);
  const int D = static_cast<int>(cfg_.d_model), KV = static_cast<int>(cfg_.kv_dim());
  const int H = static_cast<int>(cfg_.n_heads), Hkv = static_cast<int>(cfg_.n_kv_heads);
  const int hd = static_cast<int>(cfg_.head_dim());
  const AttnShape shape{B, T, H, Hkv, hd, D, KV, KV, D, 1.0f / std::sqrt(static_cast<float>(hd))};
  const size_t per_layer = static_cast<size_t>(B) * H * T * T;
  float* d_probs = nullptr;
  check_cuda(cudaMalloc(&d_probs, per_layer * 4), "attention maps buffer");
  try {
    for (size_t l = 0; l < acts_.size(); ++l) {
      attention_probs(shape, acts_[l].q, acts_[l].k, acts_[l].lse, d_probs, stream_);
      check_cuda(cudaMemcpyAsync(host_out + l * per_layer, d_probs, per_layer * 4, cudaMemcpyDeviceToHost, stream_),
                 "attention maps D2H");
      check_cuda(cudaStreamSynchronize(stream_), "attention maps");
    }
  } catch (...) {
    cudaFree(d_probs);
    throw;
  }
  cudaFree(d_probs);
  check_device("attention maps");
}

std::vector<float> Trainer::grad_norms() {
  if (grads_partial_)
    throw std::invalid_argument("the last step's gradients are sharded over the ranks (optimizer sharding)");
  const size_t n = layout_.tensors.size();
  double* d = nullptr;
  check_cuda(cudaMalloc(&d, n * sizeof(double)), "grad norms buffer");
  for (size_t i = 0; i < n; ++i)
    tensor_sumsq(G_ + layout_.tensors[i].offset, static_cast<long long>(layout_.tensors[i].numel), d + i, stream_);
  std::vector<double> h(n);
  cudaError_t e = cudaMemcpyAsync(h.data(), d, n * sizeof(double), cudaMemcpyDeviceToHost, stream_);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
  cudaFree(d);
  check_cuda(e, "grad norms");
  std::vector<float> out(n);
  for (size_t i = 0; i < n; ++i) out[i] = static_cast<float>(std::sqrt(h[i]));
  return out;
}

}  // namespace mm
