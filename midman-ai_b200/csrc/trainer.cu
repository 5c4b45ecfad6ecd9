// Trainer: buffers, parameter I/O and batch upload. The step itself is in
// trainer_step.cu.
#include "trainer.h"

#include "nccl_api.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <thread>

#include "attention.h"
#include "device.h"
#include "gemm.h"

namespace mm {

namespace {

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw std::runtime_error(std::string(what) + ": " + nccl().GetErrorString(r));
}

}  // namespace

Trainer::Trainer(const ModelConfig& cfg, int batch, int seq, int precision, int world, int rank,
                 const void* nccl_unique_id)
    : cfg_(cfg), batch_(batch), seq_(seq), precision_(precision), world_(world), rank_(rank) {
  const std::string bad = validate_config(cfg);
  if (!bad.empty()) throw std::invalid_argument(bad);
  if (batch <= 0 || seq <= 0) throw std::invalid_argument("batch and seq must be at least 1");
  if (static_cast<uint64_t>(seq) > cfg.max_seq_len)
    throw std::invalid_argument("sequence length " + std::to_string(seq) + " exceeds max_seq_len " +
                                std::to_string(cfg.max_seq_len));
  if (precision != kPrecisionTF32 && precision != kPrecision3xTF32)
    throw std::invalid_argument("precision must be 0 (TF32) or 1 (3xTF32)");
  // The tensor-memory GEMMs load rows with TMA, which needs 16-byte row strides.
  if (cfg.d_model % 4 || cfg.d_ff % 4 || cfg.vocab % 4 || cfg.kv_dim() % 4)
    throw std::invalid_argument(
        "the GPU path needs d_model, d_ff, vocab_size and n_kv_heads * head_dim to be multiples of 4");
  if (cfg.head_dim() > 128) throw std::invalid_argument("the GPU path supports head_dim up to 128");
  if (world < 1 || rank < 0 || rank >= world) throw std::invalid_argument("bad data-parallel rank/world");
  layout_ = param_layout(cfg);

  check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "stream");
  if (world_ > 1) {
    if (!nccl_unique_id) throw std::invalid_argument("data parallelism needs an NCCL unique id");
    if (const char* t = std::getenv("MIDMAN_EXCHANGE_TIMEOUT_MS"))
      if (std::atoll(t) > 0) exchange_timeout_ms_ = std::atoll(t);
    ncclUniqueId id;
    std::memcpy(&id, nccl_unique_id, sizeof(id));
    ncclComm_t comm;
    nccl_check(nccl().CommInitRank(&comm, world_, id, rank_), "ncclCommInitRank");
    comm_ = comm;
    check_cuda(cudaStreamCreateWithFlags(&comm_stream_, cudaStreamNonBlocking), "comm stream");
    layer_done_.resize(cfg.n_layers + 1);
    for (auto& e : layer_done_) check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
    check_cuda(cudaEventCreateWithFlags(&comm_done_, cudaEventDisableTiming), "event");
  }
  // per bucket: its parameters are final (updated, or broadcast by their owner)
  gathered_.resize(cfg.n_layers + 2);
  for (auto& e : gathered_) check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
  check_cuda(cudaEventCreateWithFlags(&update_done_, cudaEventDisableTiming), "event");
  buckets_ = gradient_buckets(cfg, layout_);

  auto alloc = [&](size_t bytes) {
    void* p = nullptr;
    check_cuda(cudaMalloc(&p, std::max<size_t>(bytes, 256)), "cudaMalloc");
    allocations_.push_back(p);
    return p;
  };
  auto falloc = [&](uint64_t n) { return static_cast<float*>(alloc(n * sizeof(float))); };
  const uint64_t total = layout_.total;
  P_ = falloc(total);
  G_ = falloc(total);
  M_ = falloc(total);
  V_ = falloc(total);
  check_cuda(cudaMemset(G_, 0, total * 4), "memset");
  check_cuda(cudaMemset(M_, 0, total * 4), "memset");
  check_cuda(cudaMemset(V_, 0, total * 4), "memset");

  {
    uint64_t n = 0;
    for (const TensorInfo& t : layout_.tensors) n += (t.numel + 16383) / 16384;
    d_chunks_ = static_cast<AdamChunk*>(alloc(std::max<uint64_t>(n, 1) * sizeof(AdamChunk)));
  }
  build_chunks();

  std::vector<float> cs, sn;
  rope_tables(cfg.head_dim(), cfg.max_seq_len, cfg.rope_theta, cs, sn);
  d_cos_ = falloc(cs.size());
  d_sin_ = falloc(sn.size());
  check_cuda(cudaMemcpy(d_cos_, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "rope");
  check_cuda(cudaMemcpy(d_sin_, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice), "rope");

  const uint64_t N = static_cast<uint64_t>(batch) * seq;
  const uint64_t D = cfg.d_model, F = cfg.d_ff, KV = cfg.kv_dim(), V = cfg.vocab, H = cfg.n_heads;
  d_ids_ = static_cast<int32_t*>(alloc(N * 4));
  d_tgt_ = static_cast<int32_t*>(alloc(N * 4));
  d_uniq_ = static_cast<int32_t*>(alloc(N * 4));
  d_off_ = static_cast<int32_t*>(alloc((N + 1) * 4));
  d_pos_ = static_cast<int32_t*>(alloc(N * 4));
  d_pred_ = static_cast<int32_t*>(alloc(N * 4));
  for (int slot = 0; slot < 2; ++slot)
    check_cuda(cudaMallocHost(&h_pinned_[slot], (5 * N + 1) * sizeof(int32_t)), "pinned ids");
  check_cuda(cudaMallocHost(&h_out_, 64), "pinned out");

  acts_.resize(cfg.n_layers);
  for (auto& a : acts_) {
    a.x = falloc(N * D);
    a.xn1 = falloc(N * D);
    a.rstd1 = falloc(N);
    a.q = falloc(N * D);
    a.k = falloc(N * KV);
    a.v = falloc(N * KV);
    a.o = falloc(N * D);
    a.lse = falloc(N * H);
    a.h = falloc(N * D);
    a.xn2 = falloc(N * D);
    a.rstd2 = falloc(N);
    a.g = falloc(N * F);
    a.u = falloc(N * F);
    a.act = falloc(N * F);
  }
  x_final_ = falloc(N * D);
  xf_ = falloc(N * D);
  rstdf_ = falloc(N);
  logits_ = falloc(N * V);
  row_loss_ = falloc(N);
  dx_[0] = falloc(N * D);
  dx_[1] = falloc(N * D);
  dxn_ = falloc(N * D);
  do_ = falloc(N * D);
  dq_ = falloc(N * D);
  dk_ = falloc(N * KV);
  dv_ = falloc(N * KV);
  dact_ = falloc(N * F);
  tmp_ = falloc(N * std::max(D, F));
  delta_ = falloc(N * H);
  norm_ws_ = falloc(std::max<long long>(rmsnorm_ws_floats(static_cast<int>(N), static_cast<int>(D)), 1));
  d_partials_ = static_cast<double*>(alloc(kNormBlocks * sizeof(double)));
  d_loss_ = static_cast<double*>(alloc(sizeof(double)));
  d_norm_ = falloc(4);
  {
    const int hd = static_cast<int>(cfg.head_dim());
    const AttnShape shape{batch, seq, static_cast<int>(H), static_cast<int>(cfg.n_kv_heads), hd,
                          static_cast<long long>(D), static_cast<long long>(KV), static_cast<long long>(KV),
                          static_cast<long long>(D), 1.0f};
    // TF32: fused tensor-core attention (no score buffers); 3xTF32: the tensor-core
    // form with hi/lo operands through score buffers when head_dim is 32, 64 or
    // 128, else the FP32 flash kernels
    attn_tc_ = precision == kPrecisionTF32 && attention_flash_supported(shape);
    attn_3x_ = precision == kPrecision3xTF32 && attention_tc_supported(shape);
    if (attn_3x_) attn3_ws_ = falloc(attention_3x_ws_floats(shape, static_cast<long long>(D)));
  }
  check_cuda(cudaStreamCreateWithFlags(&side_stream_, cudaStreamNonBlocking), "stream");
  check_cuda(cudaEventCreateWithFlags(&attn_side_ready_, cudaEventDisableTiming), "event");
  check_cuda(cudaEventCreateWithFlags(&attn_side_done_, cudaEventDisableTiming), "event");
  for (auto& e : side_ev_) check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
  check_cuda(cudaDeviceSynchronize(), "trainer setup");
}

Trainer::~Trainer() {
  if (stream_) cudaStreamSynchronize(stream_);
  if (comm_stream_) cudaStreamSynchronize(comm_stream_);
  if (side_stream_) cudaStreamSynchronize(side_stream_);
  for (void* p : allocations_) cudaFree(p);
  for (int32_t* p : h_pinned_)
    if (p) cudaFreeHost(p);
  if (h_out_) cudaFreeHost(h_out_);
  for (auto e : layer_done_) cudaEventDestroy(e);
  for (auto e : gathered_) cudaEventDestroy(e);
  if (update_done_) cudaEventDestroy(update_done_);
  for (auto e : prof_events_) cudaEventDestroy(e);
  if (comm_done_) cudaEventDestroy(comm_done_);
  if (comm_) nccl().CommDestroy(static_cast<ncclComm_t>(comm_));
  if (comm_stream_) cudaStreamDestroy(comm_stream_);
  if (attn_side_ready_) cudaEventDestroy(attn_side_ready_);
  if (attn_side_done_) cudaEventDestroy(attn_side_done_);
  for (auto e : side_ev_)
    if (e) cudaEventDestroy(e);
  if (side_stream_) cudaStreamDestroy(side_stream_);
  if (stream_) cudaStreamDestroy(stream_);
}

void Trainer::init_params(HostRng& rng, float init_std, int threads) {
  if (!(std::isfinite(init_std) && init_std > 0.0f)) throw std::invalid_argument("init std must be positive and finite");
  std::vector<float> host(layout_.total);
  mm::init_params(cfg_, layout_, rng, init_std, host.data(), threads);
  load_params(host.data());
}

// AdamW chunks of the range this rank updates: never across a parameter
// boundary, at most 16,384 elements; decay for rank >= 2 tensors (adamw.rs:197).
void Trainer::build_chunks() {
  const uint64_t lo = shard_begin(rank_), hi = shard_end(rank_);
  std::vector<AdamChunk> chunks;
  for (const TensorInfo& t : layout_.tensors) {
    const uint64_t b = std::max(lo, t.offset), e = std::min(hi, t.offset + t.numel);
    for (uint64_t o = b; o < e; o += 16384)
      chunks.push_back({static_cast<long long>(o), static_cast<int>(std::min<uint64_t>(16384, e - o)),
                        t.shape.size() >= 2 ? 1 : 0});
  }
  n_chunks_ = static_cast<int>(chunks.size());
  // the chunks of each bucket (buckets are unions of whole tensors; chunks come in order)
  bucket_chunks_.assign(buckets_.size(), {0, 0});
  for (size_t b = 0, c = 0; b < buckets_.size(); ++b) {
    bucket_chunks_[b].first = static_cast<int>(c);
    while (c < chunks.size() && static_cast<uint64_t>(chunks[c].offset) < buckets_[b].second) ++c;
    bucket_chunks_[b].second = static_cast<int>(c);
  }
  if (n_chunks_)
    check_cuda(cudaMemcpy(d_chunks_, chunks.data(), chunks.size() * sizeof(AdamChunk), cudaMemcpyHostToDevice),
               "chunks");
}

void Trainer::shard_optimizer(bool on) {
  if (on == zero1_) return;
  wait_params(-1);
  check_cuda(cudaStreamSynchronize(stream_), "shard optimizer");
  const uint64_t total = layout_.total;
  auto replace = [&](float*& buf, float* fresh) {
    allocations_.erase(std::find(allocations_.begin(), allocations_.end(), static_cast<void*>(buf)));
    check_cuda(cudaFree(buf), "cudaFree");
    buf = fresh;
    allocations_.push_back(fresh);
  };
  auto falloc = [&](uint64_t n) {
    void* p = nullptr;
    check_cuda(cudaMalloc(&p, std::max<uint64_t>(n * 4, 256)), "cudaMalloc");
    return static_cast<float*>(p);
  };
  if (on) {
    // ranges end on blocks of the fixed norm grid, so each block's partial is one rank's
    bounds_ = shard_bounds(total, world_, static_cast<uint64_t>(norm_block_elems(static_cast<long long>(total))),
                           kNormBlocks);
    const uint64_t lo = bounds_[rank_], n = bounds_[rank_ + 1] - lo;
    float* m = falloc(n);
    float* v = falloc(n);
    check_cuda(cudaMemcpy(m, M_ + lo, n * 4, cudaMemcpyDeviceToDevice), "shard moments");
    check_cuda(cudaMemcpy(v, V_ + lo, n * 4, cudaMemcpyDeviceToDevice), "shard moments");
    replace(M_, m);
    replace(V_, v);
    zero1_ = true;
  } else {
    float* m = falloc(total);
    float* v = falloc(total);
    gather_moment(2, 0, total, m);
    gather_moment(3, 0, total, v);
    check_cuda(cudaStreamSynchronize(stream_), "gather moments");
    replace(M_, m);
    replace(V_, v);
    zero1_ = false;
  }
  build_chunks();
}

// Copies moment `which` (2: m, 3: v) of flat elements [offset, offset + n) into a
// device buffer, each owner broadcasting its part (every rank calls this).
void Trainer::gather_moment(int which, uint64_t offset, uint64_t n, float* dst) {
  const float* src = which == 2 ? M_ : V_;
  if (!zero1_ || world_ == 1) {
    check_cuda(cudaMemcpyAsync(dst, src + offset, n * 4, cudaMemcpyDeviceToDevice, stream_), "moments");
    return;
  }
  ncclComm_t comm = static_cast<ncclComm_t>(comm_);
  nccl_check(nccl().GroupStart(), "ncclGroupStart");
  for (int r = 0; r < world_; ++r) {
    const uint64_t lo = std::max(offset, bounds_[r]), hi = std::min(offset + n, bounds_[r + 1]);
    if (lo >= hi) continue;
    const float* send = r == rank_ ? src + (lo - bounds_[r]) : dst + (lo - offset);
    nccl_check(nccl().Broadcast(send, dst + (lo - offset), hi - lo, ncclFloat, r, comm, stream_), "ncclBroadcast");
  }
  nccl_check(nccl().GroupEnd(), "ncclGroupEnd");
}

void Trainer::wait_params(int bucket) {
  if (!gather_pending_) return;
  const int last = static_cast<int>(gathered_.size()) - 1;
  check_cuda(cudaStreamWaitEvent(stream_, gathered_[bucket < 0 ? last : bucket], 0), "wait params");
  if (bucket < 0 || bucket == last) gather_pending_ = false;
}

void Trainer::load_params(const float* host) {
  wait_params(-1);
  check_cuda(cudaMemcpyAsync(P_, host, layout_.total * 4, cudaMemcpyHostToDevice, stream_), "load params");
  check_cuda(cudaStreamSynchronize(stream_), "load params");
}

void Trainer::restore(const float* params, const float* m, const float* v, uint64_t adam_steps) {
  wait_params(-1);
  const size_t bytes = layout_.total * 4;
  check_cuda(cudaMemcpyAsync(P_, params, bytes, cudaMemcpyHostToDevice, stream_), "restore params");
  // this rank's range of the moments (all of them without sharding)
  const uint64_t lo = mv_begin();
  const size_t mv_bytes = (shard_end(rank_) - lo) * 4;
  if (m) check_cuda(cudaMemcpyAsync(M_, m + lo, mv_bytes, cudaMemcpyHostToDevice, stream_), "restore moments");
  else check_cuda(cudaMemsetAsync(M_, 0, mv_bytes, stream_), "restore moments");
  if (v) check_cuda(cudaMemcpyAsync(V_, v + lo, mv_bytes, cudaMemcpyHostToDevice, stream_), "restore moments");
  else check_cuda(cudaMemsetAsync(V_, 0, mv_bytes, stream_), "restore moments");
  check_cuda(cudaStreamSynchronize(stream_), "restore");
  adam_steps_ = adam_steps;
}

void Trainer::read_params(float* host) { read_tensor(0, layout_.total, host, 0); }
void Trainer::read_grads(float* host) { read_tensor(0, layout_.total, host, 1); }

void Trainer::read_tensor(uint64_t offset, uint64_t n, float* host, int which) {
  if (offset + n > layout_.total) throw std::out_of_range("tensor range outside the parameter vector");
  if (which == 1 && grads_partial_)
    throw std::invalid_argument(
        "the last step reduced each gradient to the rank that owns it (optimizer sharding): run loss_and_grads for "
        "whole gradients");
  wait_params(-1);
  if ((which == 2 || which == 3) && zero1_ && world_ > 1) {
    // collective: the owners broadcast their parts through a device buffer, in slices
    const uint64_t slice = 1ull << 26;
    float* tmp = nullptr;
    check_cuda(cudaMalloc(&tmp, std::min(n, slice) * 4 + 256), "cudaMalloc");
    try {
      for (uint64_t o = 0; o < n; o += slice) {
        const uint64_t k = std::min(slice, n - o);
        gather_moment(which, offset + o, k, tmp);
        check_cuda(cudaMemcpyAsync(host + o, tmp, k * 4, cudaMemcpyDeviceToHost, stream_), "read tensor");
        check_cuda(cudaStreamSynchronize(stream_), "read tensor");
      }
    } catch (...) {
      cudaFree(tmp);
      throw;
    }
    check_cuda(cudaFree(tmp), "cudaFree");
    return;
  }
  const float* src = which == 0 ? P_ + offset : which == 1 ? G_ + offset : (which == 2 ? M_ : V_) + offset;
  check_cuda(cudaMemcpyAsync(host, src, n * 4, cudaMemcpyDeviceToHost, stream_), "read tensor");
  check_cuda(cudaStreamSynchronize(stream_), "read tensor");
}

void Trainer::read_moments(float* m, float* v) {
  read_tensor(0, layout_.total, m, 2);
  read_tensor(0, layout_.total, v, 3);
}

// Groups token positions by id, positions ascending within each id, so the
// embedding gradient adds rows in the reference's order (ops_shape.rs:262-272).
void Trainer::build_embedding_csr(const int32_t* inputs, int N, int slot) {
  std::vector<std::pair<int32_t, int32_t>> order(N);
  for (int i = 0; i < N; ++i) order[i] = {inputs[i], i};
  std::sort(order.begin(), order.end());
  int32_t* uniq = h_pinned_[slot] + 2 * N;
  int32_t* offs = h_pinned_[slot] + 3 * N;
  int32_t* pos = h_pinned_[slot] + 4 * N + 1;
  int nu = 0;
  for (int i = 0; i < N; ++i) {
    if (i == 0 || order[i].first != order[i - 1].first) {
      uniq[nu] = order[i].first;
      offs[nu] = i;
      ++nu;
    }
    pos[i] = order[i].second;
  }
  offs[nu] = N;
  n_uniq_slot_[slot] = nu;
}

void Trainer::upload_batch(const int32_t* inputs, const int32_t* targets, int B, int T) {
  // The previous step's copies out of slot 0 have finished: each step ends with
  // a synchronizing read of its results.
  prepare_batch(inputs, targets, B, T, 0);
  upload_prepared(0, B, T, targets != nullptr);
}

void Trainer::prepare_batch(const int32_t* inputs, const int32_t* targets, int B, int T, int slot) {
  const int N = B * T;
  if (N > batch_ * seq_) throw std::invalid_argument("batch larger than the trainer's capacity");
  if (static_cast<uint64_t>(T) > cfg_.max_seq_len) throw std::invalid_argument("sequence longer than max_seq_len");
  for (int i = 0; i < N; ++i) {
    if (inputs[i] < 0 || static_cast<uint64_t>(inputs[i]) >= cfg_.vocab)
      throw std::out_of_range("token id " + std::to_string(inputs[i]) + " is out of range for vocab " +
                              std::to_string(cfg_.vocab));
    if (targets && (targets[i] < 0 || static_cast<uint64_t>(targets[i]) >= cfg_.vocab))
      throw std::out_of_range("target class " + std::to_string(targets[i]) + " is out of range for vocab " +
                              std::to_string(cfg_.vocab));
  }
  int32_t* h = h_pinned_[slot];
  std::memcpy(h, inputs, N * 4);
  if (targets) std::memcpy(h + N, targets, N * 4);
  build_embedding_csr(inputs, N, slot);
}

void Trainer::upload_prepared(int slot, int B, int T, bool with_targets) {
  const int N = B * T;
  const int32_t* h = h_pinned_[slot];
  n_uniq_ = n_uniq_slot_[slot];
  check_cuda(cudaMemcpyAsync(d_ids_, h, N * 4, cudaMemcpyHostToDevice, stream_), "ids");
  if (with_targets) check_cuda(cudaMemcpyAsync(d_tgt_, h + N, N * 4, cudaMemcpyHostToDevice, stream_), "targets");
  check_cuda(cudaMemcpyAsync(d_uniq_, h + 2 * N, n_uniq_ * 4, cudaMemcpyHostToDevice, stream_), "uniq");
  check_cuda(cudaMemcpyAsync(d_off_, h + 3 * N, (n_uniq_ + 1) * 4, cudaMemcpyHostToDevice, stream_), "offs");
  check_cuda(cudaMemcpyAsync(d_pos_, h + 4 * N + 1, N * 4, cudaMemcpyHostToDevice, stream_), "pos");
}

void Trainer::set_profile(bool on) {
  profiling_ = on;
  profile_.clear();
  gemm_profile_.clear();
  pending_.clear();
  prof_next_ = 0;
}

int Trainer::prof_begin() {
  if (!profiling_) return -1;
  const int slot = prof_next_;
  prof_next_ += 2;
  while (static_cast<int>(prof_events_.size()) < prof_next_) {
    cudaEvent_t e;
    check_cuda(cudaEventCreate(&e), "profile event");
    prof_events_.push_back(e);
  }
  check_cuda(cudaEventRecord(prof_events_[slot], stream_), "profile event");
  return slot;
}

void Trainer::prof_end(int slot, const char* cls, double flops, std::string shape) {
  if (slot < 0) return;
  check_cuda(cudaEventRecord(prof_events_[slot + 1], stream_), "profile event");
  pending_.push_back({slot, cls, flops, std::move(shape)});
}

namespace {
void accumulate(std::vector<std::pair<std::string, Trainer::ProfileEntry>>& v, const std::string& key, float ms,
                double flops) {
  auto it = v.begin();
  for (; it != v.end(); ++it)
    if (it->first == key) break;
  if (it == v.end()) {
    v.push_back({key, Trainer::ProfileEntry{}});
    it = v.end() - 1;
  }
  it->second.launches += 1;
  it->second.ms += ms;
  it->second.flops += flops;
}
}  // namespace

// Called after the stream has synchronized.
void Trainer::prof_collect() {
  for (const Pending& p : pending_) {
    float ms = 0.0f;
    check_cuda(cudaEventElapsedTime(&ms, prof_events_[p.slot], prof_events_[p.slot + 1]), "profile elapsed");
    accumulate(profile_, p.cls, ms, p.flops);
    if (!p.shape.empty()) accumulate(gemm_profile_, p.shape, ms, p.flops);
  }
  pending_.clear();
  prof_next_ = 0;
}

void Trainer::gemm(int M, int N, int K, const float* A, long long lda, bool a_mn, const float* B, long long ldb,
                   bool b_mn, float* C, long long ldc, const float* R, long long ldr, cudaStream_t st, bool keep) {
  const GemmSegment seg{{A, lda, a_mn}, {B, ldb, b_mn}, K};
  gemm_sum(M, N, &seg, 1, C, ldc, R, ldr, st, keep);
}

// C = sum of the segments' products (+ R): one launch when the shape runs on CTA
// pairs (gemm_tf32_sum, or gemm_3xtf32_sum after the hi/lo splits).
void Trainer::gemm_sum(int M, int N, const GemmSegment* segs, int nseg, float* C, long long ldc, const float* R,
                       long long ldr, cudaStream_t st, bool keep) {
  if (!st) st = stream_;
  const int slot = st == stream_ ? prof_begin() : -1;
  DeviceContext& ctx = device_context();
  const uint64_t before = gemm_launch_count();
  int rc = 0;
  if (precision_ == kPrecisionTF32) {
    rc = gemm_tf32_sum(M, N, segs, nseg, C, ldc, R, ldr, ctx.d_err, st);
  } else {
    rc = gemm_3xtf32_sum(M, N, segs, nseg, C, ldc, R, ldr, ctx.d_err, st, &lo_cache_, keep);
    launches_ += 2 * nseg;  // the hi/lo splits of A and B
  }
  if (rc) throw std::runtime_error(std::string("GEMM: ") + gemm_status_string(rc));
  launches_ += gemm_launch_count() - before;
  if (slot >= 0) {
    double flops = 0.0;
    std::string ks;
    for (int g = 0; g < nseg; ++g) {
      flops += 2.0 * M * N * segs[g].K;
      ks += (g ? "+" : "") + std::to_string(segs[g].K);
    }
    prof_end(slot, precision_ == kPrecisionTF32 ? "gemm_tf32" : "gemm_3xtf32", flops,
             std::to_string(M) + "x" + std::to_string(N) + "x" + ks + (segs[0].a.mn_major ? " M" : " K") +
                 (segs[0].b.mn_major ? "M" : "K"));
  }
}

// With more than one rank, the wait for the step also watches the exchange: a
// peer that failed shows up as an asynchronous NCCL error, a peer that left as
// collectives that never finish. Either way the communicator is aborted (its
// kernels in flight end) after the error or the deadline, and the step fails
// with the reason; the trainer refuses further data-parallel work.
void Trainer::wait_exchange(const char* where) {
  if (world_ <= 1) return;
  if (!comm_) throw std::runtime_error(std::string(where) + ": the data-parallel exchange was aborted earlier");
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(exchange_timeout_ms_);
  for (;;) {
    const cudaError_t q = cudaStreamQuery(stream_);
    if (q == cudaSuccess) return;
    if (q != cudaErrorNotReady) check_cuda(q, where);
    ncclResult_t async = ncclSuccess;
    const ncclResult_t r = nccl().CommGetAsyncError(static_cast<ncclComm_t>(comm_), &async);
    const bool failed = r != ncclSuccess || (async != ncclSuccess && async != ncclInProgress);
    if (failed || std::chrono::steady_clock::now() >= deadline) {
      nccl().CommAbort(static_cast<ncclComm_t>(comm_));
      comm_ = nullptr;
      throw std::runtime_error(std::string(where) + ": " +
                               (failed ? std::string("NCCL reported an asynchronous error: ") +
                                             nccl().GetErrorString(r != ncclSuccess ? r : async)
                                       : "the data-parallel exchange did not finish within " +
                                             std::to_string(exchange_timeout_ms_) + " ms") +
                               "; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

void Trainer::check_device(const char* where) {
  wait_exchange(where);
  const int code = take_device_error(stream_);
  if (code) throw std::runtime_error(std::string(where) + ": " + device_error_message(code));
}

void Trainer::allreduce_grads_range(uint64_t offset, uint64_t n) {
  if (world_ <= 1 || n == 0) return;
  nccl_check(nccl().AllReduce(G_ + offset, G_ + offset, n, ncclFloat, ncclAvg, static_cast<ncclComm_t>(comm_),
                           comm_stream_),
             "ncclAllReduce(grads)");
}

// Averages bucket b's gradients on the communication stream: everywhere, or (a
// sharded update) only on the ranks owning each part of it.
void Trainer::reduce_bucket(int b) {
  const uint64_t beg = buckets_[b].first, end = buckets_[b].second;
  if (!owner_reduce_) {
    allreduce_grads_range(beg, end - beg);
    return;
  }
  ncclComm_t comm = static_cast<ncclComm_t>(comm_);
  nccl_check(nccl().GroupStart(), "ncclGroupStart");
  for (int r = 0; r < world_; ++r) {
    const uint64_t lo = std::max(beg, bounds_[r]), hi = std::min(end, bounds_[r + 1]);
    if (lo < hi)
      nccl_check(nccl().Reduce(G_ + lo, G_ + lo, hi - lo, ncclFloat, ncclAvg, r, comm, comm_stream_), "ncclReduce");
  }
  nccl_check(nccl().GroupEnd(), "ncclGroupEnd");
}

// After a sharded update: each owner broadcasts its updated parameters, bucket by
// bucket in forward order, each bucket's completion an event the next forward waits on.
void Trainer::broadcast_params() {
  check_cuda(cudaEventRecord(update_done_, stream_), "event");
  check_cuda(cudaStreamWaitEvent(comm_stream_, update_done_, 0), "wait");
  ncclComm_t comm = static_cast<ncclComm_t>(comm_);
  for (size_t b = 0; b < buckets_.size(); ++b) {
    const uint64_t beg = buckets_[b].first, end = buckets_[b].second;
    nccl_check(nccl().GroupStart(), "ncclGroupStart");
    for (int r = 0; r < world_; ++r) {
      const uint64_t lo = std::max(beg, bounds_[r]), hi = std::min(end, bounds_[r + 1]);
      if (lo < hi)
        nccl_check(nccl().Broadcast(P_ + lo, P_ + lo, hi - lo, ncclFloat, r, comm, comm_stream_), "ncclBroadcast");
    }
    nccl_check(nccl().GroupEnd(), "ncclGroupEnd");
    check_cuda(cudaEventRecord(gathered_[b], comm_stream_), "event");
  }
  gather_pending_ = true;
}

}  // namespace mm
