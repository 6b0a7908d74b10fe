// Engine::run_train on this engine: the reference device loop
// (crates/emeans-core/src/core/train.rs:60-303), restated in C++ over the
// engine's layer-1 ops. Per batch, queued without a host wait: readout
// (normalize or row norms), top-1 in chunks, scatter-add (and the closing
// sums in the last epoch), EMA. The host waits only every 5th step for the
// masses (revival plan, MT19937 on the host) and at the end. Each epoch's
// labels and scores are copied into pinned memory behind the epoch's work,
// and its statistics are computed on a helper thread while the next epoch
// runs; the closing means are computed on the device.
#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <future>
#include <string>
#include <vector>

#include "engine.h"
#include "host.h"

namespace eb {

void top1_dispatch(eb_engine* e, const Top1Args& a, eb_buf* xbuf) {
  if (top1_screen_supported(e, a))
    top1_screen(e, a, xbuf);
  else
    top1_exact(e, a);
}

namespace {

struct DevBuf {
  eb_engine* e;
  eb_buf* b;
  DevBuf(eb_engine* eng, int dtype, size_t len) : e(eng), b(new_buf(eng, dtype, len)) {}
  ~DevBuf() { free_buf(e, b); }
  float* f() { return static_cast<float*>(b->ptr); }
  uint32_t* u() { return static_cast<uint32_t*>(b->ptr); }
};

void read_into(eb_engine* e, void* dst, const void* src, size_t bytes) {
  if (bytes) EB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, e->stream));
  sync(e);
}

struct EpochStat {
  double obj, imbalance;
};

// Epoch statistics (train.rs:224-279): f64 objective per chunk, imbalance.
// With threads > 1 the batches are split into contiguous ranges summed at
// once, each batch's sum still in its own sequential order, and the batch
// sums are then added in batch order: the same bits as one thread. The
// label counts are integers (any order).
EpochStat epoch_stats(const uint32_t* lab, const float* sc, size_t rows, size_t bsz, size_t chunk,
                      size_t k, bool spherical, int threads = 1) {
  const size_t nb = (rows + bsz - 1) / bsz;
  std::vector<double> batch_obj(nb, 0.0);
  std::vector<std::vector<uint64_t>> hists(std::max(threads, 1), std::vector<uint64_t>(k, 0));
  auto part = [&](int q) {
    const size_t b0 = nb * (size_t)q / (size_t)threads, b1 = nb * (size_t)(q + 1) / (size_t)threads;
    for (size_t bi = b0; bi < b1; bi++) {
      const size_t b = bi * bsz, e = std::min(b + bsz, rows);
      double obj_batch = 0.0;
      for (size_t c0 = b; c0 < e; c0 += chunk) {
        size_t c1 = std::min(c0 + chunk, e);
        double obj = 0.0;
        if (spherical) {
          obj += 2.0 * (double)(c1 - c0);
          for (size_t i = c0; i < c1; i++) obj += (double)(-2.0f * sc[i]);
        } else {
          for (size_t i = c0; i < c1; i++) obj += (double)sc[i];
        }
        obj_batch += obj;
      }
      batch_obj[bi] = obj_batch;
    }
    std::vector<uint64_t>& hist = hists[q];
    const size_t r0 = std::min(rows, b0 * bsz), r1 = std::min(rows, b1 * bsz);
    for (size_t i = r0; i < r1; i++) {
      ensure(lab[i] < k, "device returned a label >= k");
      hist[lab[i]]++;
    }
  };
  if (threads <= 1) {
    threads = 1;
    part(0);
  } else {
    std::vector<std::future<void>> fs;
    for (int q = 1; q < threads; q++) fs.push_back(std::async(std::launch::async, part, q));
    part(0);
    for (auto& f : fs) f.get();
  }
  double obj_epoch = 0.0;
  for (size_t bi = 0; bi < nb; bi++) obj_epoch += batch_obj[bi];
  double sq = 0.0;
  for (size_t j = 0; j < k; j++) {
    uint64_t c = 0;
    for (int q = 0; q < threads; q++) c += hists[q][j];
    sq += (double)c * (double)c;
  }
  return {obj_epoch, (double)k * sq / ((double)rows * (double)rows)};
}

}  // namespace

void train(eb_engine* e, const eb_train_job* job, eb_train_out* out) {
  const size_t n = job->n, d = job->d, k = job->k;
  ensure(d > 0 && k > 0, "d and k must be positive");
  ensure(job->x != nullptr, "x is null");
  ensure(n >= k, "need at least k = " + std::to_string(k) + " rows, got " + std::to_string(n));
  ensure(out && out->centroids, "out->centroids is required");
  ensure(job->batch_law >= 0 && job->batch_law <= 2, "unknown batch law");
  ensure(!(job->state_positions == nullptr) == !(job->state_usage == nullptr),
         "state needs positions and usage");
  double tau = job->unused_threshold;
  if (std::isnan(tau)) tau = d <= 2 ? 0.0 : 0.1;
  ensure(tau >= 0.0, "unused_threshold must be >= 0 (0 disables revival)");
  const bool spherical = job->spherical != 0;
  host::Recipe r = host::resolve_recipe(n, k, d, job->nepochs, job->batch_law,
                                        (size_t)std::max<int64_t>(job->batch_size, 0),
                                        job->alpha0);
  ensure(r.epoch_rows.size() <= 64, "at most 64 epochs");
  for (size_t rows : r.epoch_rows) ensure(rows > 0, "nepochs gives an empty epoch");
  const auto t0 = std::chrono::steady_clock::now();

  // Start state (model.rs:306-349, 772-797), assembled in pinned memory on a
  // helper thread while the device buffers are set up (the initial pick
  // draws a permutation of all n rows); its upload is then a plain DMA.
  float* pos = e->pinned_get<float>("tr_pos", k * d);
  float* usage = e->pinned_get<float>("tr_usage", k);
  std::future<void> start = std::async(std::launch::async, [&] {
    if (job->state_positions) {
      std::memcpy(pos, job->state_positions, k * d * 4);
      std::memcpy(usage, job->state_usage, k * 4);
      for (size_t j = 0; j < k; j++)
        ensure(std::isfinite(usage[j]) && usage[j] >= 0.0f, "usage must be finite and >= 0");
    } else {
      std::fill(usage, usage + k, 1.0f / 65536.0f);
      if (job->init) {
        std::memcpy(pos, job->init, k * d * 4);
      } else if (n == k) {
        std::memcpy(pos, job->x, k * d * 4);
      } else {
        std::vector<uint32_t> perm = host::Mt19937(job->seed).permutation(n);
        for (size_t j = 0; j < k; j++) std::memcpy(&pos[j * d], job->x + (size_t)perm[j] * d, d * 4);
      }
      if (spherical)
        for (size_t j = 0; j < k; j++) host::normalize_row(&pos[j * d], d);
    }
    // Exponent field all ones = inf or NaN; one pass without branches.
    uint32_t nonfinite = 0;
    const uint32_t* pb = reinterpret_cast<const uint32_t*>(pos);
    for (size_t q = 0; q < k * d; q++) nonfinite |= (uint32_t)((pb[q] & 0x7f800000u) == 0x7f800000u);
    ensure(nonfinite == 0, "initial centroids must be finite");
  });

  // Events: [0, 1] epoch E's labels and scores landed in pinned set E & 1;
  // [2, 3] epoch E's order reached device buffer E & 1; [4, 5] epoch E's
  // steps finished (its order and label buffers are free again).
  struct Events {
    cudaEvent_t ev[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    ~Events() {
      for (cudaEvent_t v : ev)
        if (v) cudaEventDestroy(v);
    }
  } done;
  for (auto& v : done.ev) EB_CUDA(cudaEventCreateWithFlags(&v, cudaEventDisableTiming));
  // Per-epoch device buffers, two sets used by alternate epochs, so that an
  // epoch's order arrives and the one before's labels and scores leave while
  // the steps between run.
  DevBuf order0(e, EB_U32, n), order1(e, EB_U32, n);
  DevBuf labels0(e, EB_U32, n), labels1(e, EB_U32, n), scores0(e, EB_F32, n), scores1(e, EB_F32, n);
  uint32_t* order_d[2] = {order0.u(), order1.u()};
  uint32_t* labels_d[2] = {labels0.u(), labels1.u()};
  float* scores_d[2] = {scores0.f(), scores1.f()};
  EB_CUDA(cudaEventRecord(done.ev[4], e->stream));  // the buffers exist
  EB_CUDA(cudaEventRecord(done.ev[5], e->stream));
  // Copy streams (the engine's): `up` takes each epoch's order to the
  // device, `down` brings each epoch's labels and scores back. Declared after
  // the buffers, so that their copies have ended (the destructor waits)
  // before the buffers go.
  if (!e->copy_stream) EB_CUDA(cudaStreamCreateWithFlags(&e->copy_stream, cudaStreamNonBlocking));
  if (!e->down_stream) EB_CUDA(cudaStreamCreateWithFlags(&e->down_stream, cudaStreamNonBlocking));
  struct CopyStreams {
    cudaStream_t up, down;
    ~CopyStreams() {
      cudaStreamSynchronize(up);
      cudaStreamSynchronize(down);
    }
  } cs{e->copy_stream, e->down_stream};
  // Each epoch's permutation is drawn on a helper thread, straight into one of
  // two pinned buffers, while the previous epoch runs (the epoch-0 one while
  // the init runs; model.rs:781-784); the same thread queues its upload on
  // `up` behind the end of the epoch that last read the device buffer.
  uint32_t* h_ord[2] = {e->pinned_get<uint32_t>("tr_ord0", n), e->pinned_get<uint32_t>("tr_ord1", n)};
  const int dev = e->device;
  auto perm_of = [n, seed = job->seed, dev, &h_ord, &done, &order_d, &cs,
                  &r](size_t epoch) {
    const int par = (int)(epoch & 1);
    EB_CUDA(cudaSetDevice(dev));
    // The pinned buffer's last upload (epoch - 2) must have left it.
    if (epoch >= 2) EB_CUDA(cudaEventSynchronize(done.ev[2 + par]));
    host::Mt19937(host::epoch_seed(seed, epoch)).permutation_into(h_ord[par], n);
    EB_CUDA(cudaStreamWaitEvent(cs.up, done.ev[4 + par], 0));
    EB_CUDA(cudaMemcpyAsync(order_d[par], h_ord[par], r.epoch_rows[epoch] * 4,
                            cudaMemcpyHostToDevice, cs.up));
    EB_CUDA(cudaEventRecord(done.ev[2 + par], cs.up));
  };
  std::future<void> next_order = std::async(std::launch::async, perm_of, 0);

  const size_t bsz = r.batch_size;
  const size_t chunk = job->chunk > 0 ? (size_t)job->chunk : 65536;
  const size_t n_epochs = r.epoch_rows.size();

  // Device state (train.rs:92-101). Data bound with Assigner::bind_data
  // (the same host rows) is used in place, with its row norms and screen
  // copy; otherwise the rows are uploaded for this run.
  eb_buf* data = nullptr;
  const bool reuse = e->bound && e->bound_host == job->x && e->bound_n == n && e->bound->d == d;
  if (reuse) {
    data = e->bound;
  } else {
    int rc = eb_bind(e, job->x, n, d, &data);
    if (rc != EB_OK) throw Error(rc, eb_last_error());
  }
  struct Unbind {
    eb_engine* e;
    eb_buf* b;
    ~Unbind() {
      if (b) free_buf(e, b);
    }
  } unbind{e, reuse ? nullptr : data};
  DevBuf dpos(e, EB_F32, k * d), mass(e, EB_F32, k), readout(e, EB_F32, spherical ? k * d : k);
  DevBuf sums(e, EB_F32, k * d), counts(e, EB_U32, k), pass(e, EB_F32, k * d);
  DevBuf pairs(e, EB_U32, 2 * k);
  // Group exchange staging, one share per rank. Parity mode (group_shard
  // 0-2): the (labels, scores) slices of a batch. Reduce mode (3): the slice's
  // labels and scores, then its partial counts (k words) and sums (k x d), so
  // that one all-gather carries the step's whole exchange; offsets are
  // rounded to 4 words for 16-byte access.
  const bool reduce_mode = e->world > 1 && e->group_shard == 3;
  const size_t sh_max = (bsz + e->world - 1) / e->world;
  const size_t s4 = (sh_max + 3) / 4 * 4, k4 = (k + 3) / 4 * 4;
  const size_t share = reduce_mode ? 2 * s4 + k4 + k * d : 2 * sh_max;
  DevBuf stage(e, EB_U32, e->world > 1 ? share * e->world : 1);
  start.get();
  // The caller's result buffers are touched page by page on a helper thread
  // while the device trains (a read and a write back of one byte a page, so
  // the contents are unchanged even where a buffer aliases an input): memory
  // the caller has just allocated takes its first-touch page faults here,
  // not in the copies of the results after the last step (about 1.4 ms for
  // a C2 run's 3 MB centroids, 3 MB positions and 800 KB labels).
  std::future<void> prefault = std::async(std::launch::async, [out, k, d, n] {
    auto touch = [](void* p, size_t bytes) {
      if (!p || !bytes) return;
      volatile unsigned char* c = static_cast<volatile unsigned char*>(p);
      for (size_t o = 0; o < bytes; o += 4096) c[o] = c[o];
      c[bytes - 1] = c[bytes - 1];
    };
    touch(out->centroids, k * d * 4);
    touch(out->positions, k * d * 4);
    touch(out->usage, k * 4);
    touch(out->labels, n * 4);
  });
  EB_CUDA(cudaMemcpyAsync(dpos.f(), pos, k * d * 4, cudaMemcpyHostToDevice, e->stream));
  EB_CUDA(cudaMemcpyAsync(mass.f(), usage, k * 4, cudaMemcpyHostToDevice, e->stream));
  if (data->d == d && !data->xnorm && !spherical) {
    EB_CUDA(cudaMallocAsync(&data->xnorm, std::max<size_t>(n, 1) * 4, e->stream));
    e->device_allocs++;
    row_norms(e, static_cast<const float*>(data->ptr), n, d, data->xnorm);
  }

  host::Mt19937 split_rng(job->seed);
  // The next revival's uniforms, drawn ahead on a helper thread from
  // split_rng's current state (it changes only when a revival splits). After
  // a split, the helper starts once the next step is queued, so that the
  // device, idle while the host plans, is fed first.
  std::future<host::RevivalDraws> draws_next;
  std::unique_ptr<host::RevivalDraws> draws;
  bool draws_due = tau > 0.0;
  size_t n_splits = 0, step = 0;
  // Pinned read-backs of each epoch's labels and scores: a set of its own
  // for every epoch of runs up to 8 epochs (C2: 5 sets of 1.6 MB), else two
  // sets in turn, an epoch's copy waiting for the statistics of the epoch
  // that last read its set. Measured on C2: copies into a set the host had
  // just read (the statistics two epochs back) ran at about 4.4 GB/s instead
  // of 44, and the last epoch's held up the copy of the results behind them.
  // Then the masses and revival plan.
  const size_t nsets = n_epochs <= 8 ? n_epochs : 2;
  std::vector<uint32_t*> h_lab(nsets);
  std::vector<float*> h_sc(nsets);
  for (size_t q = 0; q < nsets; q++) {
    h_lab[q] = e->pinned_get<uint32_t>(("tr_lab" + std::to_string(q)).c_str(), n);
    h_sc[q] = e->pinned_get<float>(("tr_sc" + std::to_string(q)).c_str(), n);
  }
  // One "copies landed" event per set.
  struct SetEvents {
    std::vector<cudaEvent_t> ev;
    ~SetEvents() {
      for (cudaEvent_t v : ev)
        if (v) cudaEventDestroy(v);
    }
  } landed{std::vector<cudaEvent_t>(nsets, nullptr)};
  for (auto& v : landed.ev) EB_CUDA(cudaEventCreateWithFlags(&v, cudaEventDisableTiming));
  float* mass_h = e->pinned_get<float>("tr_mass", k);
  float* h_cent = e->pinned_get<float>("tr_cent", k * d);
  uint32_t* plan_h = e->pinned_get<uint32_t>("tr_plan", 2 * k);
  std::vector<float> mass_v(k);
  // Declared after the events, so destroyed (joined) before them.
  std::vector<std::future<void>> stats(n_epochs);
  if (out->labels)
    for (size_t i = 0; i < n; i++) out->labels[i] = -1;

  // Nonzero: the readout of dpos and the screen's summary of the next top-1's
  // centroids were made by the last EMA kernel under this generation.
  uint32_t readout_gen = 0;

  for (size_t epoch = 0; epoch < n_epochs; epoch++) {
    const size_t rows = r.epoch_rows[epoch];
    const int par = (int)(epoch & 1);
    next_order.get();  // this epoch's upload is queued
    const uint32_t* ord = h_ord[par];
    if (epoch + 1 < n_epochs) next_order = std::async(std::launch::async, perm_of, epoch + 1);
    const bool last = epoch + 1 == n_epochs;
    uint32_t* const order = order_d[par];
    uint32_t* const labels_ep = labels_d[par];
    float* const scores_ep = scores_d[par];
    EB_CUDA(cudaStreamWaitEvent(e->stream, done.ev[2 + par], 0));
    // Epoch - 2's labels and scores must have left this set of buffers.
    if (epoch >= 2) EB_CUDA(cudaStreamWaitEvent(e->stream, done.ev[par], 0));
    const size_t splits_before = n_splits;
    for (size_t b = 0; b < rows; b += bsz) {
      const size_t end = std::min(b + bsz, rows);
      // The readout: made by the last step's EMA kernel when it could (with
      // the screen's summary of the centroids), else here.
      if (!readout_gen) {
        if (spherical)
          normalize_rows(e, dpos.f(), k, d, readout.f());
        else
          row_norms(e, dpos.f(), k, d, readout.f());
      }
      // In a group, rank q scores positions [b + q s, b + (q + 1) s) of the
      // batch and the slices are all-gathered; alone, the whole batch. By
      // default (group_shard 0) a batch is split only when that shortens
      // the screen by more than the exchange costs: the screen's length in
      // centroid-tile times (the slice's row tiles spread over the SMs with
      // their centroid tiles in parts), a tile time about 0.52 µs per 64
      // columns of d (72 int8 MMAs at d = 768 take 6.2 µs), against about
      // 40 µs for the exchange (pack, all-gather, unpack, and the launch
      // chain broken around the collective; measured on two B200s, a C2
      // step with its batch split took longer than one GPU's whole step).
      // Otherwise every rank scores all of it and nothing is exchanged (the
      // same result either way).
      const size_t sh = (end - b + e->world - 1) / e->world;
      const double tile_us = 0.52 * (double)((d + 63) / 64);
      const double saved_us =
          tile_us * ((double)screen_tile_times(end - b, k, e->num_sms) -
                     (double)screen_tile_times(sh, k, e->num_sms));
      const bool split_batch =
          e->world > 1 &&
          (reduce_mode || e->group_shard == 1 || (e->group_shard == 0 && saved_us > 40.0));
      const size_t lo = split_batch ? std::min(b + (size_t)e->rank * sh, end) : b;
      const size_t hi = split_batch ? std::min(lo + sh, end) : end;
      for (size_t c0 = lo; c0 < hi; c0 += chunk) {
        Top1Args a;
        a.x = static_cast<const float*>(data->ptr);
        a.n = n;
        a.d = d;
        a.ids = order;
        a.r0 = c0;
        a.r1 = std::min(c0 + chunk, hi);
        a.c = spherical ? readout.f() : dpos.f();
        a.cnorm = spherical ? nullptr : readout.f();
        a.k = k;
        a.metric = spherical ? EB_IP : EB_L2;
        a.labels = labels_ep;
        a.scores = scores_ep;
        a.xnorm = data->xnorm;
        a.summary_gen = readout_gen;

        top1_dispatch(e, a, data);
      }
      if (reduce_mode) {
        // The north-star step: this rank's slice is scatter-added into its
        // share of the staging buffer (partial counts and sums), one
        // all-gather exchanges every rank's labels, scores and partials, and
        // every rank adds the partials in rank order (the same bits on every
        // rank for a given group size; not the single-engine row order).
        uint32_t* mine = stage.u() + (size_t)e->rank * share;
        shard_pack(e, labels_ep + lo, scores_ep + lo, hi - lo, s4, share, stage.u());
        scatter_add(e, static_cast<const float*>(data->ptr), n, d, order, lo, hi,
                    labels_ep, k, reinterpret_cast<float*>(mine + 2 * s4 + k4),
                    mine + 2 * s4, nullptr);
        group_allgather(e, stage.u(), share);
        shard_unpack(e, stage.u(), end - b, sh, s4, share, labels_ep + b, scores_ep + b);
        reduce_partials(e, stage.u(), share, e->world, 2 * s4, 2 * s4 + k4, k, d, sums.f(),
                        counts.u(), last ? pass.f() : nullptr);
      } else {
        if (split_batch) {
          shard_pack(e, labels_ep + lo, scores_ep + lo, hi - lo, sh, 2 * sh, stage.u());
          group_allgather(e, stage.u(), 2 * sh);
          shard_unpack(e, stage.u(), end - b, sh, sh, 2 * sh, labels_ep + b,
                       scores_ep + b);
        }
        scatter_add(e, static_cast<const float*>(data->ptr), n, d, order, b, end,
                    labels_ep, k, sums.f(), counts.u(), last ? pass.f() : nullptr);
      }
      const double alpha = host::scheduled_alpha(r.alpha0, step, r.total_steps);
      // The EMA step, with the next step's readout and the screen's summary
      // of the centroids it will read, in one kernel where d allows.
      readout_gen = screen_next_summary_gen(e);
      if (!ema_update_readout(e, dpos.f(), mass.f(), sums.f(), counts.u(), k, d, (float)alpha,
                              (float)(1.0 - alpha), alpha == 1.0, spherical, readout.f(),
                              screen_summary_words(e), readout_gen)) {
        readout_gen = 0;
        ema_update(e, dpos.f(), mass.f(), sums.f(), counts.u(), k, d, (float)alpha,
                   (float)(1.0 - alpha), alpha == 1.0);
      }
      if (draws_due) {
        draws_next = std::async(std::launch::async, host::revival_draws, split_rng, k);
        draws_due = false;
      }
      // Revival (a threshold of tau <= 0 marks nothing dead: no plan).
      if (tau > 0.0 && (step + 1) % 5 == 0) {
        read_into(e, mass_h, mass.f(), k * 4);
        std::memcpy(mass_v.data(), mass_h, k * 4);
        if (draws_next.valid()) draws.reset(new host::RevivalDraws(draws_next.get()));
        std::vector<uint32_t> plan = host::plan_revival(mass_v, tau, split_rng, draws.get());
        if (!plan.empty()) {
          std::memcpy(plan_h, plan.data(), plan.size() * 4);
          EB_CUDA(cudaMemcpyAsync(pairs.u(), plan_h, plan.size() * 4, cudaMemcpyHostToDevice,
                                  e->stream));
          split(e, dpos.f(), mass.f(), pairs.u(), plan.size() / 2, d);
          readout_gen = 0;  // the split moved centroids: read them out afresh
          n_splits += plan.size() / 2;
          draws.reset();  // drawn from the generator's state before this split
          draws_due = true;
        }
      }
      step++;
    }
    // Epoch end: labels and scores come down on `down` while the next epoch
    // runs; a helper thread computes the statistics once they have landed.
    EB_CUDA(cudaEventRecord(done.ev[4 + par], e->stream));
    const size_t set = epoch % nsets;
    if (epoch >= nsets) stats[epoch - nsets].get();  // the set it read is reused now
    EB_CUDA(cudaStreamWaitEvent(cs.down, done.ev[4 + par], 0));
    EB_CUDA(cudaMemcpyAsync(h_lab[set], labels_ep, rows * 4, cudaMemcpyDeviceToHost, cs.down));
    EB_CUDA(cudaMemcpyAsync(h_sc[set], scores_ep, rows * 4, cudaMemcpyDeviceToHost, cs.down));
    EB_CUDA(cudaEventRecord(landed.ev[set], cs.down));
    out->nsplit[epoch] = (int64_t)(n_splits - splits_before);
    const cudaEvent_t ev = landed.ev[set];
    const uint32_t* hl = h_lab[set];
    const float* hs = h_sc[set];
    const bool verbose = job->verbose != 0;
    if (last) prefault.get();  // the last epoch's statistics write the labels
    stats[epoch] = std::async(std::launch::async, [=]() {
      EB_CUDA(cudaSetDevice(dev));
      EB_CUDA(cudaEventSynchronize(ev));
      // The last epoch's statistics and its labels put in row order are the
      // end of the call: both run on several threads, at once. The other
      // epochs' statistics run on one thread while the device works.
      std::future<void> parts[2];
      if (last && out->labels) {
        // The captured assignments in row order, in two slices (ord is a
        // permutation: the slices write disjoint entries).
        const size_t h2 = rows / 2;
        auto place = [out, ord, hl](size_t a, size_t b) {
          for (size_t i = a; i < b; i++) out->labels[ord[i]] = (int32_t)hl[i];
        };
        parts[0] = std::async(std::launch::async, place, (size_t)0, h2);
        parts[1] = std::async(std::launch::async, place, h2, rows);
      }
      const EpochStat st = epoch_stats(hl, hs, rows, bsz, chunk, k, spherical, last ? 4 : 1);
      out->obj[epoch] = st.obj;
      out->imbalance[epoch] = st.imbalance;
      out->epoch_time[epoch] =
          std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      if (verbose)
        fprintf(stderr, "  Epoch %zu / %zu (%zu rows), iteration %zu (%.2f s): objective=%.17g\n",
                epoch + 1, n_epochs, rows, step, out->epoch_time[epoch], st.obj);
      for (auto& f : parts)
        if (f.valid()) f.get();
    });
    if (last) {
      // Closing means (core/mod.rs:404-429) on the device: the closing pass's
      // label counts, sums / count, renormalised when spherical.
      label_counts(e, labels_ep, rows, k, counts.u());
      closing_means(e, dpos.f(), pass.f(), counts.u(), k, d, sums.f());
      const float* closing = sums.f();
      if (spherical) {
        normalize_rows(e, sums.f(), k, d, pass.f());
        closing = pass.f();
      }
      EB_CUDA(cudaMemcpyAsync(h_cent, closing, k * d * 4, cudaMemcpyDeviceToHost, e->stream));
    }
  }
  // Results through pinned staging (a DMA at full speed), then into the
  // caller's buffers on four threads (each buffer in two halves).
  EB_CUDA(cudaMemcpyAsync(pos, dpos.f(), k * d * 4, cudaMemcpyDeviceToHost, e->stream));
  EB_CUDA(cudaMemcpyAsync(mass_h, mass.f(), k * 4, cudaMemcpyDeviceToHost, e->stream));
  sync(e);
  {
    const size_t half = k * d / 2;
    auto copy = [](float* dst, const float* src, size_t count) {
      std::memcpy(dst, src, count * 4);
    };
    auto c0 = std::async(std::launch::async, copy, out->centroids, h_cent, half);
    auto c1 = std::async(std::launch::async, copy, out->centroids + half, h_cent + half,
                         k * d - half);
    std::future<void> p1;
    if (out->positions) {
      p1 = std::async(std::launch::async, copy, out->positions + half, pos + half, k * d - half);
      copy(out->positions, pos, half);
    }
    if (out->usage) std::memcpy(out->usage, mass_h, k * 4);
    c0.get();
    c1.get();
    if (p1.valid()) p1.get();
  }
  for (auto& f : stats)
    if (f.valid()) f.get();
  out->n_epochs = (int32_t)n_epochs;
  out->n_splits = (int64_t)n_splits;
  out->batch_size = (int64_t)bsz;
  out->alpha0 = r.alpha0;
  out->total_steps = (int64_t)r.total_steps;
}

}  // namespace eb

extern "C" int eb_train(eb_engine* e, const eb_train_job* job, eb_train_out* out) {
  if (!e || !job || !out) {
    eb::set_last_error("engine, job and out are required");
    return EB_INVALID_ARGUMENT;
  }
  int prev = -1;
  cudaGetDevice(&prev);
  int rc = EB_OK;
  try {
    if (prev != e->device) EB_CUDA(cudaSetDevice(e->device));
    eb::train(e, job, out);
  } catch (const eb::Error& err) {
    rc = err.code;
    eb::set_last_error(err.what());
  } catch (const std::exception& err) {
    rc = EB_INTERNAL;
    eb::set_last_error(err.what());
  }
  if (prev >= 0 && prev != e->device) cudaSetDevice(prev);
  return rc;
}
