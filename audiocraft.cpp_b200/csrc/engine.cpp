// engine.cpp -- host side of libactrain.so: the C ABI of include/actrain.h.
//
// One act_ctx owns one device: the frozen base weights (f16, dequantised once from
// F32/F16/Q8_0 at bind time), the fp32 adapter master parameters with their Adam moments and
// gradient accumulator, the activation arena sized for (max_batch, frames, tokens), and one
// CUDA graph per microbatch size that replays the whole forward + backward.
//
// The schedule restates, layer by layer, the reference training graph:
//   MelodyFlow: dit_forward / dit_block (src/mf/dit.h:105-212) + MSE (src/mf/train.h:107)
//   MusicGen:   mg_train_forward (src/mg/train.h:12-49) + cross entropy (src/mg/train.h:131)
// with the backward written out explicitly (ggml autodiff in the reference,
// src/mf/train.h:118) and the optimizer of TrainAccumulation::update
// (src/ac/train_controls.h:89-118) run on the device.
#include "actrain.h"

#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "kernels.h"
#include "watchdog.h"

using namespace act;

namespace {

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define CK(x)                                                                                 \
    do {                                                                                      \
        cudaError_t e_ = (x);                                                                 \
        if (e_ != cudaSuccess) throw Error(ACT_ERR_CUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)

#define NK(x)                                                                                 \
    do {                                                                                      \
        ncclResult_t r_ = (x);                                                                \
        if (r_ != ncclSuccess) throw Error(ACT_ERR_NCCL, std::string(#x) + ": " + ncclGetErrorString(r_)); \
    } while (0)

thread_local std::string g_error;

// Host copies of a step's inputs into the pinned staging buffers, split over a few persistent
// threads and the calling one: a single thread copying the ~7 MB of a cfg-2 batch took about
// 1 ms per step, serial with the device work because the step API is synchronous.
class CopyPool {
  public:
    struct Region {
        void* dst;
        const void* src;
        size_t bytes;
    };
    explicit CopyPool(int workers) {
        for (int i = 0; i < workers; ++i) th_.emplace_back([this, i] { run(i + 1); });
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> g(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : th_) t.join();
    }
    void copy(const std::vector<Region>& regions) {
        size_t total = 0;
        for (const auto& r : regions) total += r.bytes;
        if (th_.empty() || total < (256u << 10)) {
            for (const auto& r : regions) std::memcpy(r.dst, r.src, r.bytes);
            return;
        }
        {
            std::lock_guard<std::mutex> g(mu_);
            job_ = &regions;
            total_ = total;
            remaining_ = (int)th_.size();
            ++gen_;
        }
        cv_.notify_all();
        share(0);
        std::unique_lock<std::mutex> g(mu_);
        done_.wait(g, [this] { return remaining_ == 0; });
        job_ = nullptr;
    }

  private:
    // participant p of P copies bytes [total * p / P, total * (p + 1) / P) of the regions laid end to end
    void share(int p) {
        const size_t P = th_.size() + 1, lo = total_ * p / P, hi = total_ * (p + 1) / P;
        size_t at = 0;
        for (const auto& r : *job_) {
            const size_t a = std::max(lo, at), b = std::min(hi, at + r.bytes);
            if (a < b) std::memcpy(static_cast<char*>(r.dst) + (a - at), static_cast<const char*>(r.src) + (a - at), b - a);
            at += r.bytes;
        }
    }
    void run(int p) {
        uint64_t seen = 0;
        for (;;) {
            {
                std::unique_lock<std::mutex> g(mu_);
                cv_.wait(g, [&] { return stop_ || gen_ != seen; });
                if (stop_) return;
                seen = gen_;
            }
            share(p);
            std::lock_guard<std::mutex> g(mu_);
            if (--remaining_ == 0) done_.notify_one();
        }
    }
    std::vector<std::thread> th_;
    std::mutex mu_;
    std::condition_variable cv_, done_;
    const std::vector<Region>* job_ = nullptr;
    size_t total_ = 0;
    int remaining_ = 0;
    uint64_t gen_ = 0;
    bool stop_ = false;
};

}  // namespace

void act::set_last_error(const std::string& msg) { g_error = msg; }

namespace {

const char* const kTargets[7] = {"self.qkv", "self.out", "cross.q", "cross.kv", "cross.out", "ff.0", "ff.2"};

// A frozen 2-D weight [rows = out][cols = in]: f16 (bound as F32 / F16), or a Q8_0 weight kept
// as its blocks' two fields apart: quants biased to unsigned (q + 128) [rows][cols] and f16 block
// scales transposed [cols / 32][rows].  Q8_0 weights are not expanded in HBM for the projection
// GEMMs: the GEMM's converter warps multiply quants by scales in shared memory (gemm_tc.cu).
struct Weight {
    f16* h = nullptr;
    uint8_t* q = nullptr;
    f16* d = nullptr;
    int rows = 0, cols = 0;
};

struct Proj {
    int in = 0, out = 0;
    Weight W;
    bool bound = false;
    bool adapted = false, dora = false;
    int r = 0, RP = 0;
    float s = 0.f;
    int64_t offA = 0, offB = 0, offM = -1;
    f16* A_h = nullptr;  // [RP][in], rows >= r zero
    f16* B_h = nullptr;  // [out][RP], cols >= r zero
    float* base = nullptr; // DoRA: frozen ||W_o||^2 + in*1e-12 (double accumulated on the host)
    float *P = nullptr, *G = nullptr, *Q = nullptr, *nsq = nullptr, *g = nullptr, *dg = nullptr, *scr = nullptr,
          *colpart = nullptr;
    int* colcnt = nullptr;  // dora_colsum's per-column-block counters (left at zero)
    f16* BD = nullptr;
};

struct Layer {
    Proj p[7];
    float* norm[6] = {};  // norm1.w, norm1.b, norm_cross.w, norm_cross.b, norm2.w, norm2.b
    bool consumes = false, produces = false;
    int proj = 0, src = -1;
    float *xin = nullptr, *xmid = nullptr, *xmid2 = nullptr, *xout = nullptr;
    float *mu[3] = {}, *rs[3] = {};
    f16 *h1 = nullptr, *hc = nullptr, *f = nullptr, *qkv = nullptr, *o1 = nullptr, *cq = nullptr;
    f16 *ckv = nullptr, *o2 = nullptr, *z = nullptr, *gact = nullptr;
    f16* U[7] = {};
    f16* Yaux[7] = {};
    float *lse1 = nullptr, *lse2 = nullptr;
    f16* xsave_h = nullptr;
    float* dsaved = nullptr;
};

struct PInfo {
    std::string name;
    int64_t off, rows, cols;
};

struct KStat {
    double ms = 0, flops = 0, bytes = 0;
    int64_t launches = 0;
};

}  // namespace

struct act_ctx {
    int device = 0;
    act_model_desc md{};
    act_adapter_desc ad{};
    bool mf = true;
    cudaStream_t stream = nullptr;
    // second stream for work that may overlap the main stream's (captured as graph branches)
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    bool side_pending = false;
    bool in_side = false;  // kernels are being issued on the side stream
    // stream-K workspace of the dense GEMMs (main stream only: launches sharing it must not overlap)
    float* sk_part = nullptr;
    int* sk_flag = nullptr;
    bool use_sk = true;  // ACTRAIN_STREAMK=0 at context creation: whole tiles only
    std::string err;
    bool finalized = false;
    std::vector<void*> dallocs;
    std::vector<void*> hallocs;

    int D = 0, F = 0, H = 0, L = 0, T = 0, C = 0, B = 0, RP = 0;
    int Ctok = 0;                 // the caller's conditioning tokens; C is that rounded up to 8
    int32_t* d_mgvalid = nullptr;  // MusicGen: Ctok per clip (masks the padding rows past Ctok)
    long M = 0, MC = 0;  // activation rows, context rows (capacity)

    std::vector<Layer> layers;
    // MelodyFlow globals
    Weight in_proj, out_proj, cond_w;
    float *cond_b = nullptr, *te0 = nullptr, *te2 = nullptr, *onw = nullptr, *onb = nullptr;
    std::vector<Weight> skip;
    std::vector<float> rope_ff;
    float* rope = nullptr;
    // backward gradient scale: a power of two near the loss's divisor (T * latent for the MSE,
    // scored positions for the cross entropy); seeds are multiplied by it, adapter gradients by
    // its inverse
    float gscale = 1.f, inv_gscale = 1.f;
    // MusicGen globals
    std::vector<float*> emb;
    float** emb_dev = nullptr;
    std::vector<Weight> head;
    float* pos = nullptr;
    std::map<std::string, bool> bound;

    // parameters
    int64_t nparam = 0;
    float *value = nullptr, *mom1 = nullptr, *mom2 = nullptr, *grad = nullptr;
    uint8_t* decay = nullptr;
    std::vector<PInfo> ptable;
    CopyJob* jobs_dev = nullptr;
    int njobs = 0, max_job = 0;
    double* partials = nullptr;
    int* nonfinite_dev = nullptr;
    int accumulated = 0, count_override = 0;

    // staging (host pinned + device)
    float *h_clean = nullptr, *h_noise = nullptr, *h_hidden = nullptr, *h_t = nullptr, *h_tfeat = nullptr,
          *h_loss = nullptr, *h_ctx = nullptr, *h_start = nullptr;
    int32_t *h_nvalid = nullptr, *h_ids = nullptr, *h_tgt = nullptr;
    float *d_clean = nullptr, *d_noise = nullptr, *d_hidden = nullptr, *d_t = nullptr, *d_tfeat = nullptr,
          *d_loss = nullptr, *d_ctx = nullptr, *d_start = nullptr;  // d_start: edit-bridge start, -1 = none
    float* loss_part = nullptr;  // per-clip partial sums of the MSE ([max_batch][32])
    int32_t *d_nvalid = nullptr, *d_ids = nullptr, *d_tgt = nullptr;
    float* mg_rowloss = nullptr;  // per-row cross-entropy terms of one codebook ([B][scored rows])

    // global activations / scratch
    f16 *x0 = nullptr, *hidden_h = nullptr, *ctx_h = nullptr, *xo = nullptr, *dout = nullptr, *xprev_h = nullptr;
    float *vstar = nullptr, *te1 = nullptr, *te = nullptr, *x0f = nullptr, *muo = nullptr, *rso = nullptr,
          *outp = nullptr;
    float *dx = nullptr, *dtmp = nullptr, *dq_acc = nullptr, *dvec = nullptr;
    int* dq_turn = nullptr;  // self-attention backward: ordered dQ adds ([B][H][ceil(T/128)])
    bool deterministic = false;  // act_set_deterministic: ordered dQ adds in the tcgen05 backward
    float* dkv_acc = nullptr;  // cross-attention dK | dV partials (fp32, [2][qsplit][clips * C][D])
    int cross_qsplit = 1;
    f16* dU_cond = nullptr;  // dU of cross.kv, whose gradients run on the side stream
    f16 *dxh = nullptr, *dz = nullptr, *dU = nullptr, *dob = nullptr, *dqkv = nullptr, *dcq = nullptr,
         *dckv = nullptr;
    float* logits = nullptr;
    f16* dlogits = nullptr;

    // execution
    // captured step graphs and eager-run counts, keyed by 2 * n + (1 if the step all-reduces)
    std::map<int, cudaGraphExec_t> graphs;
    std::map<int, int> eager_runs;
    std::map<int, int64_t> kernel_nodes;
    int staged_n = -1;
    bool profiling = false;
    KStat stats[3];
    struct PendingEv {
        cudaEvent_t a, b;
        int cls;
        double flops, bytes;
    };
    std::vector<PendingEv> pending;
    std::vector<cudaEvent_t> evpool;
    size_t evnext = 0;

    ncclComm_t comm = nullptr;
    // host waits on the device while a communicator is live, and NCCL initialisation, give up
    // after this long (0: no limit): the communicator is then aborted and the call fails
    int64_t timeout_ms = 0;
    // in-step gradient all-reduce (act_set_grad_sync): per-layer buckets on their own stream,
    // each started as soon as its layer's backward has been issued
    cudaStream_t comm_stream = nullptr;
    cudaEvent_t ev_comm_fork = nullptr, ev_comm_join = nullptr;
    int grad_sync = 0;               // > 0: the next step all-reduces, then averages over this count
    bool in_step_sync = false;       // the body being issued carries the all-reduce
    bool comm_pending = false;
    std::vector<std::pair<int64_t, int64_t>> layer_params;  // [first, end) of each layer's parameters
    int* kerr = nullptr;
    int* probe_flag = nullptr;  // never set: act_wait_probe waits on it until its limit runs out
    bool use_tc = true;
    // which kernel family each launch was issued to (ACT_PATH_*), counted as the step is issued
    int64_t path_count[ACT_PATH_COUNT] = {};
    // f16 expansions of Q8_0 weights, only for the generic paths (tcgen05 kernels switched off, or
    // operands neither the fused GEMM nor the rank-block kernel takes; the benchmarked steps use
    // none): two per stream, sized for the largest weight
    f16* wscratch[2][2] = {};
    long wscratch_elems = 0;
    // DoRA projections in layer order (device table for the batched factor / tail kernels) and
    // each layer's span of it
    struct DoraSpan {
        int first = 0, n = 0, max_out = 0, max_in = 0;
    };
    DoraJob* dora_jobs_dev = nullptr;
    int dora_n = 0, dora_max_out = 0;
    std::vector<DoraSpan> dora_layer;
    // The DoRA weight products and row factors depend only on the adapters and the frozen
    // weights: they run on a stream of their own, a layer ahead of the forward, which waits per
    // layer (ev_dora[l]) only for its own factors
    cudaStream_t dora_stream = nullptr;
    cudaEvent_t ev_dora_fork = nullptr;
    std::vector<cudaEvent_t> ev_dora;
    bool dora_async_ok = false;  // every P product takes the rank-block kernel (no scratch expansion)
    bool dora_async = false;     // the step being issued runs them on dora_stream

    // ------------------------------------------------------------------------------------
    template <class Tp>
    Tp* dalloc(size_t n) {
        void* p = nullptr;
        const size_t bytes = std::max<size_t>(n * sizeof(Tp), 16);
        CK(cudaMalloc(&p, bytes));
        CK(cudaMemsetAsync(p, 0, bytes, stream));
        dallocs.push_back(p);
        return static_cast<Tp*>(p);
    }
    template <class Tp>
    Tp* halloc(size_t n) {
        void* p = nullptr;
        CK(cudaMallocHost(&p, std::max<size_t>(n * sizeof(Tp), 16)));
        hallocs.push_back(p);
        return static_cast<Tp*>(p);
    }

    // ---------------------------------------------------------------- timing helpers
    cudaEvent_t next_event() {
        if (evnext >= evpool.size()) {
            cudaEvent_t e;
            CK(cudaEventCreate(&e));
            evpool.push_back(e);
        }
        return evpool[evnext++];
    }
    template <class Fn>
    void timed(int cls, double flops, double bytes, Fn&& fn) {
        if (!profiling) {
            fn();
            return;
        }
        cudaEvent_t a = next_event(), b = next_event();
        CK(cudaEventRecord(a, stream));
        fn();
        CK(cudaEventRecord(b, stream));
        pending.push_back({a, b, cls, flops, bytes});
    }
    void collect_stats() {
        if (pending.empty()) return;
        CK(cudaStreamSynchronize(stream));
        for (auto& p : pending) {
            float ms = 0;
            CK(cudaEventElapsedTime(&ms, p.a, p.b));
            stats[p.cls].ms += ms;
            stats[p.cls].flops += p.flops;
            stats[p.cls].bytes += p.bytes;
            stats[p.cls].launches += 1;
        }
        pending.clear();
        evnext = 0;
    }

    // B segment seg (1, 2) of g reads weight w from column c0: K-major (B(n, k) = w[n][c0 + k],
    // the forward) or MN-major (B(n, k) = w[k][c0 + n], the input gradient)
    static void set_b(GemmArgs& g, int seg, const Weight& w, bool kmajor, int c0 = 0) {
        g.b_kmajor = kmajor;
        const f16* h = w.h ? w.h + c0 : nullptr;
        const uint8_t* q = w.q ? w.q + c0 : nullptr;
        const f16* d = w.q ? w.d + (long)(c0 / 32) * w.rows : nullptr;
        if (seg == 1) { g.B1 = h; g.B1q = q; g.B1d = d; g.ldb1 = w.cols; g.ldd1 = w.rows; }
        else { g.B2 = h; g.B2q = q; g.B2d = d; g.ldb2 = w.cols; g.ldd2 = w.rows; }
    }
    // A Q8_0 segment that the fused path cannot take: expand its view into scratch first
    void expand_q8(GemmArgs& g) {
        for (int seg = 1; seg <= 2; ++seg) {
            const uint8_t* q = seg == 1 ? g.B1q : g.B2q;
            if (!q || (seg == 2 && g.K2 <= 0)) continue;
            const int K = seg == 1 ? g.K1 : g.K2;
            const int rows = g.b_kmajor ? g.N : K, cols = g.b_kmajor ? K : g.N;
            f16* out = wscratch[in_side ? 1 : 0][seg - 1];
            const f16* d = seg == 1 ? g.B1d : g.B2d;
            const long ldq = seg == 1 ? g.ldb1 : g.ldb2, ldd = seg == 1 ? g.ldd1 : g.ldd2;
            timed(2, 0, 0, [&] { q8_view_to_f16(q, ldq, d, ldd, rows, cols, out, cols, stream); });
            if (seg == 1) { g.B1 = out; g.B1q = nullptr; g.B1d = nullptr; g.ldb1 = cols; }
            else { g.B2 = out; g.B2q = nullptr; g.B2d = nullptr; g.ldb2 = cols; }
        }
    }

    void run_gemm(const GemmArgs& g0, int cls = 0) {
        const double fl = 2.0 * g0.M * g0.N * (double)(g0.K1 + g0.K2);
        GemmArgs g = g0;
        // stream-K only on the main stream and only while no side-stream work may run beside it:
        // its pairs wait on their neighbours, which must all be resident to finish early
        // (measured: allowing it beside the rank products costs 0.55 ms per cfg-2 step)
        if (!in_side && use_sk && !side_pending) {
            g.sk_part = sk_part;
            g.sk_flag = sk_flag;
        }
        // A few rows (a rank block, the conditioning of a small batch) run on one whole tile of
        // the tcgen05 kernel: its maps read the rows past them as zero and clip the rows written
        if (use_tc && g.M <= 128 && g.arows == 0) {
            GemmArgs t = g;
            t.arows = g.M;
            t.mvalid = std::min(g.mvalid, g.M);
            t.M = (g.B1q || (g.K2 > 0 && g.B2q)) ? 256 : 128;
            if (gemm_tc_supported(t)) g = t;
        }
        if ((g.B1q || g.B2q) && !(use_tc && gemm_tc_supported(g))) {
            expand_q8(g);
            g.a2_from_prev = false;  // the expansion now runs between A2's producer and the GEMM
        }
        if (use_tc && gemm_tc_supported(g)) {
            ++path_count[ACT_PATH_GEMM_TC];
            timed(cls, fl, 0, [&] { gemm_tc_auto(g, kerr, stream); });
        } else {
            ++path_count[ACT_PATH_GEMM_MMA];
            timed(cls, fl, 0, [&] { gemm(g, stream); });
            if (g.out_h)  // the generic path has no second output: convert afterwards
                timed(2, 0, 0, [&] {
                    residual_to_f16(static_cast<float*>(g.out), nullptr, g.out_h, nullptr, g.M, g.N, stream);
                });
        }
    }

    // Issue fn's kernels on the side stream, after everything the main stream has issued so far
    // and concurrently with what it issues until join_side().  The profiling pass keeps one
    // stream so that every launch is bracketed by its own events.
    template <class Fn>
    void on_side(Fn&& fn) {
        if (profiling) {
            fn();
            return;
        }
        CK(cudaEventRecord(ev_fork, stream));
        CK(cudaStreamWaitEvent(side, ev_fork, 0));
        std::swap(stream, side);
        in_side = true;
        fn();
        in_side = false;
        std::swap(stream, side);
        side_pending = true;
    }
    void join_side() {
        if (!side_pending) return;
        CK(cudaEventRecord(ev_join, side));
        CK(cudaStreamWaitEvent(stream, ev_join, 0));
        side_pending = false;
    }

    // In-step all-reduce of the gradient range [first, end) on the communicator's stream, after
    // everything the main stream has issued so far (that range's gradients are complete then)
    // and concurrently with what it issues next.  No-op unless this step all-reduces.
    void sync_bucket(int64_t first, int64_t end) {
        if (!in_step_sync || end <= first) return;
        CK(cudaEventRecord(ev_comm_fork, stream));
        CK(cudaStreamWaitEvent(comm_stream, ev_comm_fork, 0));
        nccl_call(ncclAllReduce(grad + first, grad + first, (size_t)(end - first), ncclFloat, ncclSum, comm,
                                comm_stream),
                  "gradient all-reduce");
        comm_pending = true;
    }
    void join_comm() {
        if (!comm_pending) return;
        CK(cudaEventRecord(ev_comm_join, comm_stream));
        CK(cudaStreamWaitEvent(stream, ev_comm_join, 0));
        comm_pending = false;
    }
    // after layer l's backward and its DoRA terms (finish_layer): its adapters' gradients are
    // final.  Layers the backward does not reach keep zero gradients on every rank.
    void sync_layer(int l) {
        if (in_step_sync) join_side();  // the layer's gA products (finish_layer) are part of it
        sync_bucket(layer_params[l].first, layer_params[l].second);
    }
    void sync_rest() {
        join_side();
        join_comm();
    }

    // rank-block products: the tcgen05 skinny kernel, or the generic GEMM `fallback` when the
    // tcgen05 paths are disabled or the operands do not qualify
    void run_rank(const SkinnyArgs& k, const GemmArgs& fallback) {
        const double fl = 2.0 * k.M * k.nb * (double)k.K;
        if (use_tc && skinny_supported(k)) {
            ++path_count[ACT_PATH_RANK_TC];
            timed(2, fl, 0, [&] { skinny_gemm(k, kerr, stream); });
        } else {
            ++path_count[ACT_PATH_RANK_MMA];
            run_gemm(fallback, 2);
        }
    }

    // ---------------------------------------------------------------- bounded waits (NCCL)
    // The communicator is gone (ncclCommAbort): graphs that carry its collectives are dropped.
    void abort_comm() {
        if (!comm) return;
        ncclCommAbort(comm);
        comm = nullptr;
        for (auto it = graphs.begin(); it != graphs.end();) {
            if (it->first & 1) {
                cudaGraphExecDestroy(it->second);
                it = graphs.erase(it);
            } else {
                ++it;
            }
        }
    }
    // Until the communicator's pending work (initialisation, an enqueue) is done: bounded by
    // timeout_ms, failure or expiry aborts it.
    void wait_nccl(const char* what) {
        const WaitResult r = bounded_wait(
            [&] {
                ncclResult_t st = ncclSuccess;
                if (ncclCommGetAsyncError(comm, &st) != ncclSuccess) return WaitState::Failed;
                return st == ncclSuccess ? WaitState::Done : st == ncclInProgress ? WaitState::Pending : WaitState::Failed;
            },
            [&] { abort_comm(); }, timeout_ms, 100);
        if (r != WaitResult::Done)
            throw Error(ACT_ERR_NCCL, std::string("NCCL ") + what + (r == WaitResult::TimedOut ? " timed out" : " failed") +
                                          ": communicator aborted");
    }
    void nccl_call(ncclResult_t r, const char* what) {
        if (r == ncclInProgress) return wait_nccl(what);
        if (r != ncclSuccess) {
            abort_comm();
            throw Error(ACT_ERR_NCCL, std::string("NCCL ") + what + ": " + ncclGetErrorString(r));
        }
    }
    // Wait for the context's stream.  While a communicator is live, a collective whose peer died
    // or stalled never finishes: poll the stream and NCCL's asynchronous error, within timeout_ms.
    void sync_stream() {
        if (!comm) {
            CK(cudaStreamSynchronize(stream));
            return;
        }
        cudaError_t cerr = cudaSuccess;
        const WaitResult r = bounded_wait(
            [&] {
                const cudaError_t e = cudaStreamQuery(stream);
                if (e == cudaSuccess) return WaitState::Done;
                if (e != cudaErrorNotReady) {
                    cerr = e;
                    return WaitState::Done;
                }
                ncclResult_t st = ncclSuccess;
                if (ncclCommGetAsyncError(comm, &st) != ncclSuccess || (st != ncclSuccess && st != ncclInProgress))
                    return WaitState::Failed;
                return WaitState::Pending;
            },
            [&] { abort_comm(); }, timeout_ms, 50);
        if (cerr != cudaSuccess) throw Error(ACT_ERR_CUDA, std::string("stream: ") + cudaGetErrorString(cerr));
        if (r != WaitResult::Done) {
            // after the abort the collective returns and the stream drains
            cudaStreamSynchronize(stream);
            throw Error(ACT_ERR_NCCL, r == WaitResult::TimedOut
                                          ? "timed out waiting for a collective (a peer rank stalled or died): communicator aborted"
                                          : "NCCL reported an asynchronous error: communicator aborted");
        }
    }

    // kernels record a nonzero code here instead of hanging on a wait that cannot finish
    // (the word is cleared when it is reported, so that the context stays usable afterwards)
    void check_kernel_error() {
        int e = 0;
        CK(cudaMemcpyAsync(&e, kerr, sizeof(int), cudaMemcpyDeviceToHost, stream));
        sync_stream();
        if (e) {
            CK(cudaMemsetAsync(kerr, 0, sizeof(int), stream));
            CK(cudaStreamSynchronize(stream));
            throw Error(ACT_ERR_CUDA, "device kernel reported a timed-out wait (code " + std::to_string(e) + ")");
        }
    }

    // split-K count for the token reductions: about two CTAs per SM, each with a long enough
    // run of 64-deep k-tiles to keep its pipeline full and its final atomics rare
    static int splitk_for(long tiles, long ktiles) {
        long s = std::max<long>(1, 296 / std::max<long>(tiles, 1));
        s = std::min<long>(s, std::max<long>(1, ktiles / 8));
        return (int)std::min<long>(s, 64);
    }

    // ---------------------------------------------------------------- projections
    // Y = (X W^T + s (X A^T) B^T) * g  with the epilogue given in `e` (mode/out/ldo/resid/aux).
    void proj_fwd(Proj& p, const f16* X, long rows, f16* U, GemmArgs e) {
        if (p.adapted) {
            GemmArgs u;
            u.M = (int)rows; u.N = p.RP; u.K1 = p.in;
            u.A1 = X; u.lda1 = p.in; u.B1 = p.A_h; u.ldb1 = p.in;
            u.mode = EPI_STORE_F16; u.alpha = p.s; u.out = U; u.ldo = p.RP;
            SkinnyArgs k;  // U = s X A^T
            k.M = (int)rows; k.K = p.in; k.nb = p.RP;
            k.A = X; k.lda = p.in; k.B = p.A_h; k.ldb = p.in;
            k.kind = SKINNY_STORE; k.alpha = p.s; k.out = U; k.ldo = p.RP;
            run_rank(k, u);
        }
        e.M = (int)rows; e.N = p.out; e.K1 = p.in;
        e.A1 = X; e.lda1 = p.in; set_b(e, 1, p.W, true);
        if (p.adapted) {
            e.K2 = p.RP; e.A2 = U; e.lda2 = p.RP; e.B2 = p.B_h; e.ldb2 = p.RP;
            e.a2_from_prev = true;  // U was written by the launch just above
        }
        if (p.dora) e.colscale = p.g;
        run_gemm(e, 0);
    }

    // Adapter gradients of one projection from dYl (= dY * g, f16 [rows][out]) and, when
    // `e` has an output, the input gradient dX = dYl W + dU A.
    // inline_grads: dB / dA run on the current stream and nothing is joined (the caller has put
    // the whole call on the side stream); dUb: the dU scratch (default: the main one)
    void proj_bwd(Proj& p, const f16* dYl, long rows, const f16* X, const f16* U, const f16* Y,
                  bool want_dx, GemmArgs e, f16* dUb = nullptr, bool inline_grads = false) {
        f16* const dUs = dUb ? dUb : dU;
        if (p.dora)
            timed(2, 0, 4.0 * rows * p.out,
                  [&] { dora_colsum(dYl, p.out, Y, p.out, (int)rows, p.out, p.g, p.dg, p.colpart, p.colcnt, inv_gscale, stream); });
        if (p.adapted) {
            GemmArgs u;
            u.M = (int)rows; u.N = p.RP; u.K1 = p.out;
            u.A1 = dYl; u.lda1 = p.out; u.B1 = p.B_h; u.ldb1 = p.RP; u.b_kmajor = false;
            u.mode = EPI_STORE_F16; u.alpha = p.s; u.out = dUs; u.ldo = p.RP;
            SkinnyArgs ku;  // dU = s dYl B
            ku.M = (int)rows; ku.K = p.out; ku.nb = p.RP;
            ku.A = dYl; ku.lda = p.out; ku.B = p.B_h; ku.ldb = p.RP; ku.b_mn = true;
            ku.kind = SKINNY_STORE; ku.alpha = p.s; ku.out = dUs; ku.ldo = p.RP;
            run_rank(ku, u);
            GemmArgs gb;
            gb.M = p.out; gb.N = p.RP; gb.K1 = (int)rows;
            gb.A1 = dYl; gb.lda1 = p.out; gb.a_kmajor = false;
            gb.B1 = U; gb.ldb1 = p.RP; gb.b_kmajor = false;
            gb.mode = EPI_ATOMIC_F32; gb.alpha = inv_gscale; gb.out = grad + p.offB; gb.ldo = p.r; gb.nvalid = p.r;
            gb.splitk = splitk_for((long)((p.out + 63) / 64), (rows + 63) / 64);
            SkinnyArgs kb;  // dB += dYl^T U   ([out][r])
            kb.M = p.out; kb.K = (int)rows; kb.nb = p.r;
            kb.A = dYl; kb.lda = p.out; kb.a_mn = true; kb.B = U; kb.ldb = p.RP; kb.b_mn = true;
            kb.kind = SKINNY_ACC; kb.alpha = inv_gscale; kb.out = grad + p.offB; kb.ldo = p.r;
            GemmArgs ga;
            ga.M = p.RP; ga.N = p.in; ga.K1 = (int)rows;
            ga.A1 = dUs; ga.lda1 = p.RP; ga.a_kmajor = false;
            ga.B1 = X; ga.ldb1 = p.in; ga.b_kmajor = false;
            ga.mode = EPI_ATOMIC_F32; ga.alpha = inv_gscale; ga.out = grad + p.offA; ga.ldo = p.in; ga.mvalid = p.r;
            ga.splitk = splitk_for((long)((p.in + 127) / 128), (rows + 63) / 64);
            SkinnyArgs ka;  // dA += dU^T X   ([r][in], computed as its transpose)
            ka.M = p.in; ka.K = (int)rows; ka.nb = p.r;
            ka.A = X; ka.lda = p.in; ka.a_mn = true; ka.B = dUs; ka.ldb = p.RP; ka.b_mn = true;
            ka.kind = SKINNY_ACC_T; ka.alpha = inv_gscale; ka.out = grad + p.offA; ka.ldo = p.in;
            // the adapter gradients only read dYl, U, X and dU: they overlap the input-gradient
            // GEMM below (which fills its last wave with idle SMs) and join before returning
            if (inline_grads) {
                run_rank(kb, gb);
                run_rank(ka, ga);
            } else {
                on_side([&] {
                    run_rank(kb, gb);
                    run_rank(ka, ga);
                });
            }
        }
        if (!want_dx) {
            if (!inline_grads) join_side();
            return;
        }
        e.M = (int)rows; e.N = p.in; e.K1 = p.out;
        e.A1 = dYl; e.lda1 = p.out; set_b(e, 1, p.W, false);
        if (p.adapted) {
            e.K2 = p.RP; e.A2 = dUs; e.lda2 = p.RP; e.B2 = p.A_h; e.ldb2 = p.in;
            e.a2_from_prev = true;  // dU: the last launch on this stream (dB / dA went to the side)
        }
        run_gemm(e, 0);
        join_side();
    }

    // ---------------------------------------------------------------- the step
    // The large operand of a rank-block product that is a whole frozen weight W [out][in]
    // (A(m, k) = W[m][k], or W[k][m] with mn): its f16 values, or its Q8_0 quants and scales,
    // which the kernel dequantises on the way into the MMA
    static void set_rank_weight(SkinnyArgs& k, const Weight& w, bool mn) {
        k.a_mn = mn;
        k.lda = w.cols;
        if (w.q) { k.Aq = w.q; k.Ad = w.d; k.ldad = w.rows; }
        else k.A = w.h;
    }
    // The same product on the generic GEMM (tcgen05 paths off, or operands the rank-block kernel
    // does not take): the weight's f16 view, expanded into this stream's scratch if quantised
    void run_rank_weight(const SkinnyArgs& k, const Weight& w, GemmArgs fallback, bool a_is_w) {
        if (use_tc && skinny_supported(k)) {
            ++path_count[ACT_PATH_RANK_TC];
            timed(2, 2.0 * k.M * k.nb * (double)k.K, 0, [&] { skinny_gemm(k, kerr, stream); });
            return;
        }
        const f16* Wh = w.h;
        if (!Wh) {
            f16* out = wscratch[in_side ? 1 : 0][0];
            timed(2, 0, 0, [&] { q8_view_to_f16(w.q, w.cols, w.d, w.rows, w.rows, w.cols, out, w.cols, stream); });
            Wh = out;
        }
        if (a_is_w) fallback.A1 = Wh;
        else fallback.B1 = Wh;
        ++path_count[ACT_PATH_RANK_MMA];
        run_gemm(fallback, 2);
    }

    // P = W A^T [out][RP]: a rank-block product reading the frozen weight once (kept quantised:
    // the kernel's converter warps dequantise it)
    void dora_p_product(Proj& p) {
        SkinnyArgs k;
        k.M = p.out; k.K = p.in; k.nb = p.RP;
        set_rank_weight(k, p.W, false);
        k.B = p.A_h; k.ldb = p.in;
        k.kind = SKINNY_ACC; k.alpha = 1.0f; k.out = p.P; k.ldo = p.RP;
        GemmArgs a;
        a.M = p.out; a.N = p.RP; a.K1 = p.in;
        a.lda1 = p.in; a.B1 = p.A_h; a.ldb1 = p.in;
        a.mode = EPI_STORE_F32; a.out = p.P; a.ldo = p.RP;
        if (use_tc && skinny_supported(k)) CK(cudaMemsetAsync(p.P, 0, sizeof(float) * p.out * p.RP, stream));
        run_rank_weight(k, p.W, a, true);
    }

    void prepare_adapters() {
        timed(2, 0, 0, [&] { refresh_f16(jobs_dev, njobs, max_job, stream); });
        dora_async = dora_n > 0 && dora_async_ok && use_tc && !profiling;
        if (dora_async) {
            CK(cudaEventRecord(ev_dora_fork, stream));
            CK(cudaStreamWaitEvent(dora_stream, ev_dora_fork, 0));
            std::swap(stream, dora_stream);
            for (size_t l = 0; l < layers.size(); ++l) {
                for (auto& p : layers[l].p)
                    if (p.dora) dora_p_product(p);
                const DoraSpan& sp = dora_layer[l];
                if (sp.n) dora_factors(dora_jobs_dev + sp.first, sp.n, ad.rank, sp.max_out, stream);
                CK(cudaEventRecord(ev_dora[l], stream));
            }
            std::swap(stream, dora_stream);
            return;
        }
        for (auto& lay : layers)
            for (auto& p : lay.p)
                if (p.dora) dora_p_product(p);
        // the row factors of every DoRA projection in one pass per stage
        if (dora_n)
            timed(2, 0, 0, [&] { dora_factors(dora_jobs_dev, dora_n, ad.rank, dora_max_out, stream); });
    }

    // DoRA terms of layer l's adapter gradients, once its backward has been issued (its column
    // sums dg are complete then: only its own projections add into them)
    void finish_layer(int l) {
        const DoraSpan& sp = dora_layer[l];
        if (!sp.n) return;
        timed(2, 0, 0, [&] {
            dora_tail(dora_jobs_dev + sp.first, sp.n, ad.rank, sp.max_out, sp.max_in, gscale, stream);
        });
        // gA += BD^T W, as (W^T BD)^T over the out dimension: only adds into gA, so it runs on
        // the side stream beside the next layer's backward (joined before the all-reduce of this
        // layer and at the end of the step)
        on_side([&] {
            for (auto& p : layers[l].p) {
                if (!p.dora) continue;
                SkinnyArgs k;
                k.M = p.in; k.K = p.out; k.nb = p.r;
                set_rank_weight(k, p.W, true);
                k.B = p.BD; k.ldb = p.RP; k.b_mn = true;
                k.kind = SKINNY_ACC_T; k.alpha = inv_gscale; k.out = grad + p.offA; k.ldo = p.in;
                GemmArgs a;
                a.M = p.RP; a.N = p.in; a.K1 = p.out;
                a.A1 = p.BD; a.lda1 = p.RP; a.a_kmajor = false;
                a.ldb1 = p.in; a.b_kmajor = false;
                a.mode = EPI_ATOMIC_F32; a.alpha = inv_gscale; a.out = grad + p.offA; a.ldo = p.in; a.mvalid = p.r;
                a.splitk = splitk_for((p.in + 127) / 128, (p.out + 63) / 64);
                run_rank_weight(k, p.W, a, false);
            }
        });
    }

    // One transformer block forward.  te: per-clip timestep embedding (MelodyFlow) or null.
    void block_fwd(int l, int n, const int* nvalid_dev) {
        Layer& y = layers[l];
        if (dora_async) CK(cudaStreamWaitEvent(stream, ev_dora[l], 0));  // this layer's DoRA factors
        const long rows = (long)n * T, crows = (long)n * C;
        const float eps = md.norm_eps;
        const bool dit = mf;
        // the cross-attention K/V projection reads only the conditioning: it runs on the side
        // stream, overlapping the self-attention half of the block
        on_side([&] {
            GemmArgs k; k.mode = EPI_STORE_F16; k.out = y.ckv; k.ldo = 2 * D;
            proj_fwd(y.p[3], ctx_h, crows, y.U[3], k);
        });
        // pre-norm self-attention
        timed(2, 0, 0, [&] { layernorm_fwd(y.xin, y.norm[0], y.norm[1], dit ? te : nullptr, T, y.h1, y.mu[0], y.rs[0], (int)rows, D, eps, stream); });
        {
            // q and k leave the projection already rotated (RoPE in the epilogue); DoRA keeps the
            // unrotated output for its row-norm gradient
            GemmArgs e; e.mode = EPI_STORE_F16; e.out = y.qkv; e.ldo = 3 * D;
            if (dit) { e.rope = rope; e.rope_T = T; e.rope_cols = 2 * D; }
            if (y.p[0].dora) { e.aux = y.Yaux[0]; e.ldaux = 3 * D; }
            proj_fwd(y.p[0], y.h1, rows, y.U[0], e);
        }
        AttnArgs sa;
        sa.q = y.qkv; sa.k = y.qkv + D; sa.v = y.qkv + 2 * D; sa.ldq = sa.ldk = sa.ldv = 3 * D;
        sa.T = T; sa.Tk = T; sa.H = H; sa.clips = n; sa.causal = dit ? 0 : 1; sa.zero_key = dit ? md.add_zero_attn : 0;
        sa.rope = dit ? rope : nullptr; sa.rope_load = 0; sa.scale = 1.0f / std::sqrt((float)md.head_dim);
        sa.o = y.o1; sa.ldo = D; sa.lse = y.lse1;
        const bool fwd_tc = use_tc && attn_fwd_tc_supported(sa);
        ++path_count[fwd_tc ? ACT_PATH_ATTN_FWD_TC : ACT_PATH_ATTN_FWD_MMA];
        timed(1, attn_flops(n, T, true), 0, [&] {
            if (fwd_tc) attn_fwd_tc(sa, kerr, stream);
            else attn_fwd(sa, stream);
        });
        {
            GemmArgs e; e.mode = EPI_RESID_F32; e.out = y.xmid; e.ldo = D; e.resid = y.xin; e.ldr = D;
            if (y.p[1].dora) { e.aux = y.Yaux[1]; e.ldaux = D; }
            proj_fwd(y.p[1], y.o1, rows, y.U[1], e);
        }
        // cross-attention
        timed(2, 0, 0, [&] { layernorm_fwd(y.xmid, y.norm[2], y.norm[3], dit ? te : nullptr, T, y.hc, y.mu[1], y.rs[1], (int)rows, D, eps, stream); });
        {
            GemmArgs e; e.mode = EPI_STORE_F16; e.out = y.cq; e.ldo = D;
            proj_fwd(y.p[2], y.hc, rows, y.U[2], e);
        }
        join_side();
        AttnArgs ca;
        ca.q = y.cq; ca.ldq = D; ca.k = y.ckv; ca.v = y.ckv + D; ca.ldk = ca.ldv = 2 * D;
        ca.T = T; ca.Tk = C; ca.H = H; ca.clips = n; ca.nvalid = dit ? nvalid_dev : (C != Ctok ? d_mgvalid : nullptr);
        ca.zero_key = dit ? md.add_zero_attn : 0; ca.scale = sa.scale;
        ca.o = y.o2; ca.ldo = D; ca.lse = y.lse2;
        const bool xfwd_tc = use_tc && xattn_tc_supported(ca);
        ++path_count[xfwd_tc ? ACT_PATH_XATTN_FWD_TC : ACT_PATH_ATTN_FWD_MMA];
        timed(1, attn_flops(n, C, false), 0, [&] {
            if (xfwd_tc) xattn_fwd_tc(ca, kerr, stream);
            else attn_fwd(ca, stream);
        });
        {
            GemmArgs e; e.mode = EPI_RESID_F32; e.out = y.xmid2; e.ldo = D; e.resid = y.xmid; e.ldr = D;
            if (y.p[4].dora) { e.aux = y.Yaux[4]; e.ldaux = D; }
            proj_fwd(y.p[4], y.o2, rows, y.U[4], e);
        }
        // feed-forward (no timestep)
        timed(2, 0, 0, [&] { layernorm_fwd(y.xmid2, y.norm[4], y.norm[5], nullptr, T, y.f, y.mu[2], y.rs[2], (int)rows, D, eps, stream); });
        {
            // ff.0 stores its pre-activation z; the activation runs by table as its own pass
            // (the GEMM epilogue is then a plain store).  Without DoRA on ff.0 the backward needs
            // only gelu'(z), which replaces z in place.
            if (y.p[5].dora) {
                GemmArgs e; e.mode = EPI_GELU; e.out = y.gact; e.ldo = F; e.aux = y.z; e.ldaux = F;
                proj_fwd(y.p[5], y.f, rows, y.U[5], e);
            } else {
                GemmArgs e; e.mode = EPI_STORE_F16; e.out = y.z; e.ldo = F;
                proj_fwd(y.p[5], y.f, rows, y.U[5], e);
                timed(2, 0, 6.0 * rows * F, [&] { gelu_fwd(y.z, y.gact, rows * F, 1, stream); });
            }
            // the layer output also in f16 where a skip projection reads it: as this layer's saved
            // copy (a skip source) or as the next layer's x_prev operand
            GemmArgs o; o.mode = EPI_RESID_F32; o.out = y.xout; o.ldo = D; o.resid = y.xmid2; o.ldr = D;
            o.out_h = y.produces ? y.xsave_h : (writes_prev_bf(l) ? xprev_h : nullptr);
            if (y.p[6].dora) { o.aux = y.Yaux[6]; o.ldaux = D; }
            proj_fwd(y.p[6], y.gact, rows, y.U[6], o);
        }
    }

    // block l's ff.2 epilogue leaves f16(xout) in xprev_h for the skip projection of block l+1
    bool writes_prev_bf(int l) const { return !layers[l].produces && l + 1 < L && layers[l + 1].consumes; }

    // Backward of block l.  On entry dx/dxh hold d(loss)/d(xout) (dxh already scaled by
    // the DoRA factor of ff.2).  On exit dx holds d(loss)/d(xin) and dxh is NOT prepared.
    // need_dx_in: the gradient of the block's input is needed (accumulated into dx by the last
    // norm's backward, which also writes dxh = f16((dx + cvt_extra) * cvt_scale) when cvt is
    // set: the operand of whatever consumes dx next, without a separate conversion pass)
    void block_bwd(int l, int n, const int* nvalid_dev, bool need_dx_in, bool cvt = false,
                   const float* cvt_extra = nullptr, const float* cvt_scale = nullptr) {
        Layer& y = layers[l];
        const long rows = (long)n * T, crows = (long)n * C;
        const bool dit = mf;
        // ---- feed-forward
        {
            GemmArgs e; e.mode = y.p[5].dora ? EPI_GELU_BWD : EPI_GELU_BWD_D; e.out = dz; e.ldo = F; e.auxin = y.z; e.ldauxin = F;
            e.colscale2 = y.p[5].dora ? y.p[5].g : nullptr;
            proj_bwd(y.p[6], dxh, rows, y.gact, y.U[6], y.Yaux[6], true, e);
            GemmArgs d; d.mode = EPI_STORE_F32; d.out = dtmp; d.ldo = D;
            proj_bwd(y.p[5], dz, rows, y.f, y.U[5], y.z, true, d);
        }
        timed(2, 0, 0, [&] { layernorm_bwd(dtmp, y.xmid2, y.norm[4], y.mu[2], y.rs[2], dx, 1, nullptr, dxh, y.p[4].dora ? y.p[4].g : nullptr, (int)rows, D, stream); });
        // ---- cross-attention
        {
            GemmArgs e; e.mode = EPI_STORE_F16; e.out = dob; e.ldo = D;
            proj_bwd(y.p[4], dxh, rows, y.o2, y.U[4], y.Yaux[4], true, e);
        }
        AttnArgs ca;
        ca.q = y.cq; ca.ldq = D; ca.k = y.ckv; ca.v = y.ckv + D; ca.ldk = ca.ldv = 2 * D;
        ca.T = T; ca.Tk = C; ca.H = H; ca.clips = n; ca.nvalid = dit ? nvalid_dev : (C != Ctok ? d_mgvalid : nullptr);
        ca.zero_key = dit ? md.add_zero_attn : 0; ca.scale = 1.0f / std::sqrt((float)md.head_dim);
        ca.o = y.o2; ca.ldo = D; ca.lse = y.lse2;
        ca.dout = dob; ca.lddo = D; ca.dvec = dvec; ca.dq_acc = dq_acc; ca.ldq_acc = D;
        // dK / dV of the conditioning only feed an adapter on cross.kv (the conditioning itself
        // takes no gradient): without one they are not computed
        const bool need_dkv = y.p[3].adapted;
        if (need_dkv) {
            ca.dk = dckv; ca.dv = dckv + D; ca.lddk = ca.lddv = 2 * D;
        }
        ca.kscale = y.p[3].dora ? y.p[3].g : nullptr; ca.vscale = y.p[3].dora ? y.p[3].g + D : nullptr;
        // few keys: split every (head, clip)'s query blocks over CTAs, dK / dV through fp32 partials
        const bool split = C <= 64;
        if (split) {
            ca.qsplit = cross_qsplit;
            if (need_dkv) {
                ca.dk_acc = dkv_acc;
                ca.dv_acc = dkv_acc + (long)cross_qsplit * crows * D;
            }
        }
        // a single key block: each query row's dQ is final in one CTA and goes straight to dcq as
        // f16 (no fp32 accumulator to clear or convert)
        const bool dq_direct = C <= 64;
        if (dq_direct) {
            ca.dq_h = dcq;
            ca.lddq_h = D;
            ca.dq_scale = y.p[2].dora ? y.p[2].g : nullptr;
        }
        // at most 64 keys: the query-major tcgen05 backward (softmax recomputed, no dvec pass)
        const bool xbwd_tc = use_tc && dq_direct && xattn_bwd_tc_supported(ca);
        ++path_count[xbwd_tc ? ACT_PATH_XATTN_BWD_TC : ACT_PATH_ATTN_BWD_MMA];
        timed(1, 2 * attn_flops(n, C, false), 0, [&] {
            if (xbwd_tc) {
                xattn_bwd_tc(ca, kerr, stream);  // adds the dK / dV slices itself
                return;
            }
            if (!dq_direct) CK(cudaMemsetAsync(dq_acc, 0, sizeof(float) * rows * D, stream));
            attn_bwd(ca, stream);
            if (split && need_dkv) attn_dkv_finish(ca, stream);
            if (!dq_direct) attn_dq_finish(ca, dcq, D, y.p[2].dora ? y.p[2].g : nullptr, stream);
        });
        // cross.kv's adapter gradients (the conditioning needs no input gradient) go to the side
        // stream with their own dU scratch: they overlap cross.q's backward, and the join after
        // its input-gradient GEMM collects them before anything reads them
        if (need_dkv)
            on_side([&] { proj_bwd(y.p[3], dckv, crows, ctx_h, y.U[3], y.ckv, false, GemmArgs(), dU_cond, true); });
        {
            GemmArgs e; e.mode = EPI_STORE_F32; e.out = dtmp; e.ldo = D;
            proj_bwd(y.p[2], dcq, rows, y.hc, y.U[2], y.cq, true, e);
        }
        timed(2, 0, 0, [&] { layernorm_bwd(dtmp, y.xmid, y.norm[2], y.mu[1], y.rs[1], dx, 1, nullptr, dxh, y.p[1].dora ? y.p[1].g : nullptr, (int)rows, D, stream); });
        // ---- self-attention
        {
            GemmArgs e; e.mode = EPI_STORE_F16; e.out = dob; e.ldo = D;
            proj_bwd(y.p[1], dxh, rows, y.o1, y.U[1], y.Yaux[1], true, e);
        }
        AttnArgs sa;
        sa.q = y.qkv; sa.k = y.qkv + D; sa.v = y.qkv + 2 * D; sa.ldq = sa.ldk = sa.ldv = 3 * D;
        sa.T = T; sa.Tk = T; sa.H = H; sa.clips = n; sa.causal = dit ? 0 : 1; sa.zero_key = dit ? md.add_zero_attn : 0;
        sa.rope = dit ? rope : nullptr; sa.rope_load = 0; sa.scale = ca.scale;
        sa.o = y.o1; sa.ldo = D; sa.lse = y.lse1;
        sa.dout = dob; sa.lddo = D; sa.dvec = dvec; sa.dq_acc = dq_acc; sa.ldq_acc = D;
        sa.dq_turn = deterministic ? dq_turn : nullptr;
        sa.dk = dqkv + D; sa.dv = dqkv + 2 * D; sa.lddk = sa.lddv = 3 * D;
        sa.kscale = y.p[0].dora ? y.p[0].g + D : nullptr; sa.vscale = y.p[0].dora ? y.p[0].g + 2 * D : nullptr;
        const bool bwd_tc = use_tc && attn_bwd_tc_supported(sa);
        ++path_count[bwd_tc ? ACT_PATH_ATTN_BWD_TC : ACT_PATH_ATTN_BWD_MMA];
        timed(1, 2 * attn_flops(n, T, true), 0, [&] {
            CK(cudaMemsetAsync(dq_acc, 0, sizeof(float) * rows * D, stream));
            if (bwd_tc && sa.dq_turn) CK(cudaMemsetAsync(dq_turn, 0, sizeof(int) * n * H * ((T + 127) / 128), stream));
            if (bwd_tc) attn_bwd_tc(sa, kerr, stream);
            else attn_bwd(sa, stream);
            attn_dq_finish(sa, dqkv, 3 * D, y.p[0].dora ? y.p[0].g : nullptr, stream);
        });
        {
            GemmArgs e; e.mode = EPI_STORE_F32; e.out = dtmp; e.ldo = D;
            proj_bwd(y.p[0], dqkv, rows, y.h1, y.U[0], y.p[0].dora ? y.Yaux[0] : y.qkv, need_dx_in, e);
        }
        if (need_dx_in)
            timed(2, 0, 0, [&] {
                layernorm_bwd(dtmp, y.xin, y.norm[0], y.mu[0], y.rs[0], dx, 1, cvt ? cvt_extra : nullptr,
                              cvt ? dxh : nullptr, cvt ? cvt_scale : nullptr, (int)rows, D, stream);
            });
    }

    double attn_flops(int n, int keys, bool self) const {
        const double tk = keys + ((mf && md.add_zero_attn) ? 1 : 0);
        double f = 4.0 * n * T * tk * D;
        if (self && !mf) f = 4.0 * n * (T * (T + 1.0) / 2.0) * D;  // causal
        return f;
    }

    // dxh := f16((dx + dsaved[l]) * g_ff2(l))  -- entering block l's backward
    const float* entry_extra(int l) { return layers[l].produces ? layers[l].dsaved : nullptr; }
    const float* entry_scale(int l) { return layers[l].p[6].dora ? layers[l].p[6].g : nullptr; }
    void prepare_dxh(int l, int n) {
        const long rows = (long)n * T;
        timed(2, 0, 0, [&] { residual_to_f16(dx, entry_extra(l), dxh, entry_scale(l), (int)rows, D, stream); });
    }

    void mf_graph_body(int n) {
        const long rows = (long)n * T, crows = (long)n * C;
        prepare_adapters();
        timed(2, 0, 0, [&] {
            mf_inputs(d_clean, d_noise, d_t, d_start, n, T, md.latent_dim, x0, vstar, stream);
            linear_f32(d_tfeat, te0, te1, n, D, md.time_dim, 1, stream);
            linear_f32(te1, te2, te, n, D, D, 0, stream);
            f32_to_f16(d_hidden, hidden_h, crows * md.cond_dim, stream);
        });
        {
            GemmArgs c;  // context = hidden cond_proj^T + bias
            c.M = (int)crows; c.N = D; c.K1 = md.cond_dim; c.A1 = hidden_h; c.lda1 = md.cond_dim;
            set_b(c, 1, cond_w, true); c.mode = EPI_BIAS_F16; c.bias = cond_b; c.out = ctx_h; c.ldo = D;
            run_gemm(c, 0);
            GemmArgs x;  // in_proj
            x.M = (int)rows; x.N = D; x.K1 = md.latent_dim; x.A1 = x0; x.lda1 = md.latent_dim;
            set_b(x, 1, in_proj, true); x.mode = EPI_STORE_F32; x.out = x0f; x.ldo = D;
            run_gemm(x, 0);
        }
        for (int l = 0; l < L; ++l) {
            Layer& y = layers[l];
            if (y.consumes) {
                if (!writes_prev_bf(l - 1))
                    timed(2, 0, 0, [&] { residual_to_f16(layers[l - 1].xout, nullptr, xprev_h, nullptr, (int)rows, D, stream); });
                GemmArgs k;
                k.M = (int)rows; k.N = D; k.K1 = D; k.K2 = D;
                k.A1 = xprev_h; k.lda1 = D; k.A2 = layers[y.src].xsave_h; k.lda2 = D;
                set_b(k, 1, skip[y.proj], true); set_b(k, 2, skip[y.proj], true, D);
                k.mode = EPI_STORE_F32; k.out = y.xin; k.ldo = D;
                run_gemm(k, 0);
            }
            block_fwd(l, n, d_nvalid);
        }
        Layer& last = layers[L - 1];
        timed(2, 0, 0, [&] { layernorm_fwd(last.xout, onw, onb, nullptr, T, xo, muo, rso, (int)rows, D, md.norm_eps, stream); });
        {
            GemmArgs o;
            o.M = (int)rows; o.N = md.latent_dim; o.K1 = D; o.A1 = xo; o.lda1 = D; set_b(o, 1, out_proj, true);
            o.mode = EPI_STORE_F32; o.out = outp; o.ldo = md.latent_dim;
            run_gemm(o, 0);
        }
        timed(2, 0, 0, [&] { mf_loss(outp, vstar, n, T, md.latent_dim, d_loss, dout, loss_part, gscale, stream); });
        // ---------------- backward
        {
            GemmArgs d;
            d.M = (int)rows; d.N = D; d.K1 = md.latent_dim; d.A1 = dout; d.lda1 = md.latent_dim;
            set_b(d, 1, out_proj, false); d.mode = EPI_STORE_F32; d.out = dtmp; d.ldo = D;
            run_gemm(d, 0);
        }
        timed(2, 0, 0, [&] {
            for (auto& y : layers)
                if (y.produces) CK(cudaMemsetAsync(y.dsaved, 0, sizeof(float) * rows * D, stream));
            // also block L-1's entry operand dxh (see block_bwd's cvt)
            layernorm_bwd(dtmp, last.xout, onw, muo, rso, dx, 0, entry_extra(L - 1), dxh, entry_scale(L - 1),
                          (int)rows, D, stream);
        });
        const int first = ad.first_layer;
        for (int l = L - 1; l >= first; --l) {
            Layer& y = layers[l];
            const bool need_dx = l > first, via_skip = need_dx && y.consumes;
            // the block's last norm backward writes the next operand: f16(dx) for the skip
            // projection, else block l-1's entry operand
            if (via_skip) block_bwd(l, n, d_nvalid, need_dx, true, nullptr, nullptr);
            else if (need_dx) block_bwd(l, n, d_nvalid, need_dx, true, entry_extra(l - 1), entry_scale(l - 1));
            else block_bwd(l, n, d_nvalid, need_dx);
            if (via_skip) {
                GemmArgs a;  // d x_prev = dx Wskip[:, :D]
                a.M = (int)rows; a.N = D; a.K1 = D; a.A1 = dxh; a.lda1 = D;
                set_b(a, 1, skip[y.proj], false); a.mode = EPI_STORE_F32; a.out = dx; a.ldo = D;
                run_gemm(a, 0);
                GemmArgs b = a;  // d saved += dx Wskip[:, D:]
                set_b(b, 1, skip[y.proj], false, D); b.mode = EPI_ACCUM_F32; b.out = layers[y.src].dsaved;
                run_gemm(b, 0);
                prepare_dxh(l - 1, n);
            }
            finish_layer(l);
            sync_layer(l);
        }
        sync_rest();
    }

    void mg_graph_body(int n) {
        const long rows = (long)n * T, crows = (long)n * C;
        const int frames = ad.frames, prefix = ad.prefix_frames, nq = md.n_q, card = md.card;
        const int sel = frames - prefix;
        prepare_adapters();
        timed(2, 0, 0, [&] {
            mg_embed(d_ids, T, nq, emb_dev, pos, x0f, D, n, stream);
            f32_to_f16(d_ctx, ctx_h, crows * D, stream);
        });
        for (int l = 0; l < L; ++l) block_fwd(l, n, nullptr);
        Layer& last = layers[L - 1];
        timed(2, 0, 0, [&] {
            layernorm_fwd(last.xout, onw, onb, nullptr, T, xo, muo, rso, (int)rows, D, md.norm_eps, stream);
            CK(cudaMemsetAsync(d_loss, 0, sizeof(float) * n, stream));
            CK(cudaMemsetAsync(dtmp, 0, sizeof(float) * rows * D, stream));
        });
        // The head per codebook over every row of every sample (src/mg/train.h:131-140 scores
        // rows q + prefix .. q + frames - 1 of each sequence for codebook q): one logits GEMM,
        // one cross-entropy over the scored rows, one input-gradient GEMM.  Codebook q's
        // [B][T][card] block sits at a fixed place (maximum batch), so a row of dlogits is scored
        // or not whatever the microbatch: the unscored rows stay zero from allocation and add
        // nothing to the input gradient.
        const float inv_nsel = 1.0f / (float)(nq * sel);
        for (int q = 0; q < nq; ++q) {
            float* lg = logits + (long)q * B * T * card;
            f16* dl = dlogits + (long)q * B * T * card;
            GemmArgs hgm;
            hgm.M = (int)rows; hgm.N = card; hgm.K1 = D; hgm.A1 = xo; hgm.lda1 = D;
            set_b(hgm, 1, head[q], true); hgm.mode = EPI_STORE_F32; hgm.out = lg; hgm.ldo = card;
            run_gemm(hgm, 0);
            timed(2, 0, 0, [&] {
                mg_cross_entropy(lg, n, sel, T, q + prefix, card, d_tgt + (long)q * sel, (long)nq * sel, inv_nsel,
                                 d_loss, mg_rowloss, dl, gscale, stream);
            });
            GemmArgs dg;
            dg.M = (int)rows; dg.N = D; dg.K1 = card; dg.A1 = dl; dg.lda1 = card;
            set_b(dg, 1, head[q], false);
            dg.mode = EPI_ACCUM_F32; dg.out = dtmp; dg.ldo = D;
            run_gemm(dg, 0);
        }
        timed(2, 0, 0, [&] {
            layernorm_bwd(dtmp, last.xout, onw, muo, rso, dx, 0, entry_extra(L - 1), dxh, entry_scale(L - 1),
                          (int)rows, D, stream);
        });
        const int first = ad.first_layer;
        for (int l = L - 1; l >= first; --l) {
            if (l > first) block_bwd(l, n, nullptr, true, true, entry_extra(l - 1), entry_scale(l - 1));
            else block_bwd(l, n, nullptr, false);
            finish_layer(l);
            sync_layer(l);
        }
        sync_rest();
    }

    void run_body(int n) {
        if (mf) mf_graph_body(n);
        else mg_graph_body(n);
    }

    void launch_step(int n) {
        if (profiling) {
            run_body(n);
            CK(cudaGetLastError());
            collect_stats();
            return;
        }
        const int key = 2 * n + (in_step_sync ? 1 : 0);
        auto it = graphs.find(key);
        if (it == graphs.end()) {
            if (eager_runs[key]++ == 0) {  // first use of this size runs eagerly (sets kernel attributes)
                run_body(n);
                CK(cudaGetLastError());
                return;
            }
            cudaGraph_t graph;
            CK(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
            try {
                run_body(n);
            } catch (...) {
                cudaStreamEndCapture(stream, &graph);
                throw;
            }
            CK(cudaStreamEndCapture(stream, &graph));
            size_t nn = 0;
            CK(cudaGraphGetNodes(graph, nullptr, &nn));
            std::vector<cudaGraphNode_t> nodes(nn);
            CK(cudaGraphGetNodes(graph, nodes.data(), &nn));
            int64_t kn = 0;
            for (auto nd : nodes) {
                cudaGraphNodeType ty;
                CK(cudaGraphNodeGetType(nd, &ty));
                kn += ty == cudaGraphNodeTypeKernel;
            }
            kernel_nodes[n] = kn;  // the step's graph (with the all-reduce's kernels when it carries them)
            cudaGraphExec_t exec;
            CK(cudaGraphInstantiate(&exec, graph, 0));
            CK(cudaGraphDestroy(graph));
            it = graphs.emplace(key, exec).first;
        }
        CK(cudaGraphLaunch(it->second, stream));
    }

    // ---------------------------------------------------------------- staging
    std::unique_ptr<CopyPool> copies;
    CopyPool& copy_pool() {
        if (!copies) {
            const unsigned hc = std::thread::hardware_concurrency();
            copies.reset(new CopyPool((int)std::min(7u, hc > 1 ? hc - 1 : 0u)));
        }
        return *copies;
    }

    // Caller arrays -> pinned staging -> device, in pieces of about 1.5 MB: each piece's copy to
    // the device runs while the host copies the next one (the host copy and the host-to-device
    // transfer of a cfg-2 batch each take about half a millisecond).
    struct Upload {
        void* dev;
        void* pinned;
        const void* src;
        size_t bytes;
    };
    void upload(const std::vector<Upload>& ups) {
        constexpr size_t PIECE = 3u << 19;
        for (const auto& u : ups)
            for (size_t off = 0; off < u.bytes; off += PIECE) {
                const size_t len = std::min(PIECE, u.bytes - off);
                copy_pool().copy({{static_cast<char*>(u.pinned) + off, static_cast<const char*>(u.src) + off, len}});
                CK(cudaMemcpyAsync(static_cast<char*>(u.dev) + off, static_cast<char*>(u.pinned) + off, len,
                                   cudaMemcpyHostToDevice, stream));
            }
    }

    // n clips of `rows` host rows each into the device's `padded`-row layout (zero rows after)
    void upload_rows(void* dev, void* pinned, const void* src, int n, int rows, int padded, size_t row_bytes) {
        if (rows == padded) {
            upload({{dev, pinned, src, (size_t)n * rows * row_bytes}});
            return;
        }
        char* p = static_cast<char*>(pinned);
        for (int i = 0; i < n; ++i) {
            std::memcpy(p + (size_t)i * padded * row_bytes, static_cast<const char*>(src) + (size_t)i * rows * row_bytes,
                        (size_t)rows * row_bytes);
            std::memset(p + ((size_t)i * padded + rows) * row_bytes, 0, (size_t)(padded - rows) * row_bytes);
        }
        CK(cudaMemcpyAsync(dev, pinned, (size_t)n * padded * row_bytes, cudaMemcpyHostToDevice, stream));
    }

    void stage_mf(const act_mf_batch* b) {
        if (!mf) throw Error(ACT_ERR_INVALID, "not a MelodyFlow context");
        const bool bridge = b && b->pivot, sampled = b && b->stddev;
        if (!b || b->n <= 0 || b->n > B || !b->clean || (bridge && !b->edit_start) || (!bridge && !sampled && !b->noise) ||
            (bridge && sampled) || !b->hidden || !b->t)
            throw Error(ACT_ERR_INVALID, "invalid training sample");
        const int n = b->n, lat = md.latent_dim;
        const size_t nx = (size_t)n * lat * T;
        for (int i = 0; i < n; ++i) {
            const float t = b->t[i];
            if (!std::isfinite(t) || t < 0 || t > 1) throw Error(ACT_ERR_INVALID, "invalid training sample");
            // src/mf/train.h:193-195
            const float start = bridge ? b->edit_start[i] : -1.0f;
            if (bridge && (!std::isfinite(start) || start < 0 || start >= 1 || t < start))
                throw Error(ACT_ERR_INVALID, "invalid edit bridge");
            h_start[i] = start;
            const int v = b->valid_tokens ? b->valid_tokens[i] : -1;
            if (v > Ctok) throw Error(ACT_ERR_INVALID, "invalid valid token count");
            const bool uncond = b->unconditional && b->unconditional[i];
            h_nvalid[i] = uncond ? 0 : (v >= 0 ? v : Ctok);
            h_t[i] = t;
            // timestep features on the host, float arithmetic as src/ac/transformer.h:144-154
            const int half = md.time_dim / 2;
            float* tf = h_tfeat + (size_t)i * md.time_dim;
            for (int k = 0; k < md.time_dim; ++k) tf[k] = 0.f;
            for (int k = 0; k < half; ++k) {
                const float freq = std::exp(-std::log(10000.0f) * (float)k / (float)half);
                const float arg = t * freq;
                tf[k] = std::cos(arg);
                tf[half + k] = std::sin(arg);
            }
        }
        // the bridge's pivot takes the noise buffer: the input kernel turns it into the endpoint
        // on-device sampling: mean and stddev go up in place of clean and noise, then are drawn from
        upload({{d_clean, h_clean, b->clean, nx * 4},
                {d_noise, h_noise, bridge ? b->pivot : sampled ? b->stddev : b->noise, nx * 4}});
        if (sampled) mf_sample(d_clean, d_noise, n, (long)lat * T, b->sample_seed, b->window0, stream);
        upload_rows(d_hidden, h_hidden, b->hidden, n, Ctok, C, (size_t)md.cond_dim * 4);
        CK(cudaMemcpyAsync(d_t, h_t, n * 4, cudaMemcpyHostToDevice, stream));
        CK(cudaMemcpyAsync(d_start, h_start, n * 4, cudaMemcpyHostToDevice, stream));
        CK(cudaMemcpyAsync(d_tfeat, h_tfeat, (size_t)n * md.time_dim * 4, cudaMemcpyHostToDevice, stream));
        CK(cudaMemcpyAsync(d_nvalid, h_nvalid, n * 4, cudaMemcpyHostToDevice, stream));
        staged_n = n;
    }

    void stage_mg(const act_mg_batch* b) {
        if (mf) throw Error(ACT_ERR_INVALID, "not a MusicGen context");
        if (!b || b->n <= 0 || b->n > B || !b->codes || !b->context)
            throw Error(ACT_ERR_INVALID, "invalid training sample shape");
        const int n = b->n, nq = md.n_q, frames = ad.frames, prefix = ad.prefix_frames, sel = frames - prefix;
        const int S = 1 + frames + (nq - 1);  // src/mg/pattern.h:55
        for (size_t i = 0; i < (size_t)n * nq * frames; ++i)
            if (b->codes[i] < 0 || b->codes[i] >= md.card) throw Error(ACT_ERR_INVALID, "invalid codec token");
        for (size_t i = 0; i < (size_t)n * Ctok * D; ++i)
            if (!std::isfinite(b->context[i])) throw Error(ACT_ERR_INVALID, "nonfinite condition");
        for (int s = 0; s < n; ++s) {
            const int32_t* codes = b->codes + (size_t)s * nq * frames;
            for (int q = 0; q < nq; ++q) {
                // build_pattern_sequence (src/mg/pattern.h:64-76), inputs = seq[:, :S-1]
                for (int st = 0; st < T; ++st) {
                    const int t = st - 1 - q;  // delays[q] = q
                    h_ids[((size_t)s * nq + q) * T + st] = (st > 0 && t >= 0 && t < frames) ? codes[(size_t)q * frames + t]
                                                                                             : md.special_token_id;
                }
                for (int k = 0; k < sel; ++k) h_tgt[((size_t)s * nq + q) * sel + k] = codes[(size_t)q * frames + prefix + k];
            }
        }
        (void)S;
        CK(cudaMemcpyAsync(d_ids, h_ids, (size_t)n * nq * T * 4, cudaMemcpyHostToDevice, stream));
        CK(cudaMemcpyAsync(d_tgt, h_tgt, (size_t)n * nq * sel * 4, cudaMemcpyHostToDevice, stream));
        upload_rows(d_ctx, h_ctx, b->context, n, Ctok, C, (size_t)D * 4);
        staged_n = n;
    }

    void run_staged(float* loss) {
        if (!finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        if (staged_n <= 0) throw Error(ACT_ERR_STATE, "no staged batch");
        const int n = staged_n;
        in_step_sync = grad_sync > 0;
        if (in_step_sync && !comm) throw Error(ACT_ERR_STATE, "in-step gradient all-reduce needs a communicator");
        try {
            launch_step(n);
        } catch (...) {
            in_step_sync = false;
            throw;
        }
        accumulated += n;
        if (in_step_sync) {  // the step's all-reduce replaced a separate act_allreduce_grads call
            count_override = grad_sync;
            grad_sync = 0;
            in_step_sync = false;
        }
        if (loss) {
            CK(cudaMemcpyAsync(h_loss, d_loss, n * 4, cudaMemcpyDeviceToHost, stream));
            check_kernel_error();
            for (int i = 0; i < n; ++i) {
                if (!std::isfinite(h_loss[i])) throw Error(ACT_ERR_NONFINITE, "nonfinite training loss");
                loss[i] = h_loss[i];
            }
        }
    }

    // ---------------------------------------------------------------- setup
    void setup(int dev, const act_model_desc* m, const act_adapter_desc* a) {
        device = dev;
        md = *m;
        ad = *a;
        mf = md.family == ACT_FAMILY_MELODYFLOW;
        if (md.family != ACT_FAMILY_MELODYFLOW && md.family != ACT_FAMILY_MUSICGEN)
            throw Error(ACT_ERR_INVALID, "unknown model family");
        if (md.dim != md.heads * md.head_dim) throw Error(ACT_ERR_INVALID, "dim does not equal heads * head_dim");
        if (md.head_dim != 64) throw Error(ACT_ERR_INVALID, "the attention kernels need head_dim 64");
        if (md.dim % 128 || md.dim > 2048 || md.ff_dim % 128) throw Error(ACT_ERR_INVALID, "dim and ff_dim must be multiples of 128 (dim <= 2048)");
        if (mf && md.n_skip != (md.layers - 1) / 2)
            throw Error(ACT_ERR_INVALID, "DiT skip count does not match (layers - 1) / 2");
        if (!mf && md.special_token_id != md.card) throw Error(ACT_ERR_INVALID, "special_token_id should be card");
        if (ad.frames <= 0 || ad.tokens <= 0 || ad.rank <= 0 || ad.rank > md.dim || !std::isfinite(ad.alpha) ||
            ad.alpha <= 0 || ad.first_layer < 0 || ad.first_layer >= md.layers ||
            (ad.type != ACT_ADAPTER_LORA && ad.type != ACT_ADAPTER_DORA_ROWS) || ad.max_batch <= 0 ||
            (ad.targets & ~0x7Fu) || !ad.targets)
            throw Error(ACT_ERR_INVALID, "invalid training dimensions or adapter configuration");
        if (!mf && (ad.prefix_frames < 0 || ad.prefix_frames >= ad.frames))
            throw Error(ACT_ERR_INVALID, "invalid MusicGen training configuration");
        if (mf && (md.latent_dim % 8 || md.cond_dim % 8 || md.time_dim % 2))
            throw Error(ACT_ERR_INVALID, "latent_dim and cond_dim must be multiples of 8");
        CK(cudaSetDevice(device));
        CK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        CK(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking));
        CK(cudaEventCreateWithFlags(&ev_fork, cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&ev_join, cudaEventDisableTiming));
        CK(cudaStreamCreateWithFlags(&comm_stream, cudaStreamNonBlocking));
        CK(cudaEventCreateWithFlags(&ev_comm_fork, cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&ev_comm_join, cudaEventDisableTiming));
        kerr = dalloc<int>(1);
        probe_flag = dalloc<int>(1);
        {
            int sms = 0;
            CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
            sk_part = dalloc<float>(gemm_sk_part_floats(sms));
            sk_flag = dalloc<int>(gemm_sk_flag_count(sms));
        }
        const char* skv = std::getenv("ACTRAIN_STREAMK");
        use_sk = !(skv && std::string(skv) == "0");
        const char* gp = std::getenv("ACTRAIN_GEMM");
        use_tc = !(gp && std::string(gp) == "mma");
        D = md.dim; F = md.ff_dim; H = md.heads; L = md.layers;
        // the conditioning is padded to a multiple of 8 rows on the device; the rows past the
        // caller's tokens are masked in cross-attention (MelodyFlow already masks past
        // valid_tokens; MusicGen attends to all of the caller's rows, zero padding included, as
        // src/mg/train.h:181-186 does, and to none of ours)
        Ctok = ad.tokens; C = (Ctok + 7) / 8 * 8; B = ad.max_batch;
        T = mf ? ad.frames : ad.frames + md.n_q - 1;  // MusicGen: pattern steps - 1 (src/mg/train.h:74)
        RP = (ad.rank + 31) / 32 * 32;
        {
            // gradient scale: the power of two nearest the loss's divisor, so that the scaled
            // seed gradient is O(1) (an exact power of two: unscaling adds no rounding)
            const double divisor = mf ? (double)T * md.latent_dim : (double)md.n_q * (ad.frames - ad.prefix_frames);
            gscale = std::ldexp(1.0f, (int)std::lround(std::log2(std::max(divisor, 1.0))));
            inv_gscale = 1.0f / gscale;
        }
        M = (long)B * T;
        MC = (long)B * C;
        layers.resize(L);
        int sp = 0;
        std::vector<int> stack;
        for (int l = 0; l < L; ++l) {
            Layer& y = layers[l];
            if (mf) {  // dit_skip_plan, src/mf/dit.h:87-100
                const double half = (double)L / 2.0;
                y.consumes = md.n_skip > 0 && (double)l > half;
                y.produces = md.n_skip > 0 && (double)l < half - 1.0;
                if (y.consumes) {
                    if (stack.empty()) throw Error(ACT_ERR_INVALID, "DiT skip stack underflow");
                    y.proj = l % md.n_skip;
                    y.src = stack.back();
                    stack.pop_back();
                }
                if (y.produces) stack.push_back(l);
            }
            for (int t = 0; t < 7; ++t) {
                Proj& p = y.p[t];
                p.in = t == 6 ? F : D;
                p.out = t == 0 ? 3 * D : t == 3 ? 2 * D : t == 5 ? F : D;
            }
        }
        (void)sp;
    }

    // GGUF name -> binding
    void bind(const char* cname, int type, const void* host, size_t bytes) {
        if (finalized) throw Error(ACT_ERR_STATE, "weights are bound before act_finalize");
        if (!cname || !host) throw Error(ACT_ERR_INVALID, "null weight");
        const std::string name = cname;
        long rows = 0, cols = 0;
        enum { DST_F16, DST_F32, DST_HOST } dst_kind = DST_F16;
        void** dst = nullptr;    // fp32 destinations
        Weight* wdst = nullptr;  // 2-D weights (f16 or Q8_0)
        Proj* proj = nullptr;
        const std::string pre = mf ? "dit." : "lm.";
        auto layer_of = [&](const std::string& rest, int& l, std::string& tail) {
            const size_t dot = rest.find('.');
            if (dot == std::string::npos) return false;
            for (size_t i = 0; i < dot; ++i)
                if (!isdigit((unsigned char)rest[i])) return false;
            l = std::stoi(rest.substr(0, dot));
            tail = rest.substr(dot + 1);
            return l >= 0 && l < L;
        };
        std::vector<float> f32;  // host fp32 copy when needed
        if (name.rfind(pre, 0) != 0) throw Error(ACT_ERR_INVALID, "unexpected tensor: " + name);
        const std::string rest = name.substr(pre.size());
        int l = -1;
        std::string tail;
        if (layer_of(rest, l, tail)) {
            Layer& y = layers[l];
            static const char* norms[6] = {"norm1.weight", "norm1.bias", "norm_cross.weight", "norm_cross.bias",
                                           "norm2.weight", "norm2.bias"};
            for (int i = 0; i < 6; ++i)
                if (tail == norms[i]) { dst = (void**)&y.norm[i]; dst_kind = DST_F32; rows = 1; cols = D; }
            for (int t = 0; t < 7; ++t)
                if (tail == std::string(kTargets[t]) + ".weight") {
                    proj = &y.p[t];
                    wdst = &proj->W;
                    rows = proj->out;
                    cols = proj->in;
                }
        } else if (mf) {
            if (rest == "in_proj.weight") { wdst = &in_proj; rows = D; cols = md.latent_dim; }
            else if (rest == "out_proj.weight") { wdst = &out_proj; rows = md.latent_dim; cols = D; }
            else if (rest == "time_embed.0.weight") { dst = (void**)&te0; dst_kind = DST_F32; rows = D; cols = md.time_dim; }
            else if (rest == "time_embed.2.weight") { dst = (void**)&te2; dst_kind = DST_F32; rows = D; cols = D; }
            else if (rest == "cond_proj.weight") { wdst = &cond_w; rows = D; cols = md.cond_dim; }
            else if (rest == "cond_proj.bias") { dst = (void**)&cond_b; dst_kind = DST_F32; rows = 1; cols = D; }
            else if (rest == "out_norm.weight") { dst = (void**)&onw; dst_kind = DST_F32; rows = 1; cols = D; }
            else if (rest == "out_norm.bias") { dst = (void**)&onb; dst_kind = DST_F32; rows = 1; cols = D; }
            else if (rest == "rope_freq_factors") { dst_kind = DST_HOST; rows = 1; cols = md.head_dim / 2; }
            else if (rest.rfind("skip.", 0) == 0) {
                const int i = std::atoi(rest.c_str() + 5);
                if (i < 0 || i >= md.n_skip || rest != "skip." + std::to_string(i) + ".weight")
                    throw Error(ACT_ERR_INVALID, "unexpected tensor: " + name);
                wdst = &skip[i]; rows = D; cols = 2 * D;
            } else if (rest == "latent_mean" || rest == "latent_std" || rest == "time_embed.0.bias") {
                return;  // cache normalisation: not used by the step
            }
        } else {
            if (rest == "out_norm.weight") { dst = (void**)&onw; dst_kind = DST_F32; rows = 1; cols = D; }
            else if (rest == "out_norm.bias") { dst = (void**)&onb; dst_kind = DST_F32; rows = 1; cols = D; }
            else if (rest.rfind("emb.", 0) == 0 || rest.rfind("head.", 0) == 0) {
                const bool isemb = rest[0] == 'e';
                const int q = std::atoi(rest.c_str() + (isemb ? 4 : 5));
                if (q < 0 || q >= md.n_q) throw Error(ACT_ERR_INVALID, "unexpected tensor: " + name);
                if (isemb) { dst = (void**)&emb[q]; dst_kind = DST_F32; rows = md.card + 1; cols = D; }
                else { wdst = &head[q]; rows = md.card; cols = D; }
            } else if (rest.rfind("cond_proj", 0) == 0) {
                return;  // the trainer consumes already projected conditioning
            }
        }
        if (!dst && !wdst && dst_kind != DST_HOST) throw Error(ACT_ERR_INVALID, "unexpected tensor: " + name);
        const long n = rows * cols;
        size_t need = 0;
        if (type == ACT_TYPE_F32) need = (size_t)n * 4;
        else if (type == ACT_TYPE_F16) need = (size_t)n * 2;
        else if (type == ACT_TYPE_Q8_0) {
            if (cols % 32) throw Error(ACT_ERR_INVALID, "Q8_0 rows must hold whole blocks: " + name);
            need = (size_t)n / 32 * 34;
        } else throw Error(ACT_ERR_INVALID, "unsupported weight type for " + name);
        if (bytes != need) throw Error(ACT_ERR_INVALID, "weight size mismatch: " + name);
        if (bound.count(name)) throw Error(ACT_ERR_INVALID, "weight bound twice: " + name);
        // host fp32 view (DoRA norms, fp32 destinations, rope factors)
        const bool dora_proj = proj && ad.type == ACT_ADAPTER_DORA_ROWS;
        if (dst_kind != DST_F16 || dora_proj) {
            f32.resize(n);
            if (type == ACT_TYPE_F32) std::memcpy(f32.data(), host, n * 4);
            else if (type == ACT_TYPE_F16) {
                const uint16_t* h = static_cast<const uint16_t*>(host);
                for (long i = 0; i < n; ++i) f32[i] = half_to_float(h[i]);
            } else {
                const uint8_t* blk = static_cast<const uint8_t*>(host);
                for (long bidx = 0; bidx < n / 32; ++bidx) {
                    const float d = half_to_float((uint16_t)(blk[bidx * 34] | blk[bidx * 34 + 1] << 8));
                    for (int i = 0; i < 32; ++i) f32[bidx * 32 + i] = d * (float)(int8_t)blk[bidx * 34 + 2 + i];
                }
            }
        }
        if (dst_kind == DST_HOST) {
            rope_ff = f32;
        } else if (dst_kind == DST_F32) {
            float* d = dalloc<float>(n);
            CK(cudaMemcpyAsync(d, f32.data(), n * 4, cudaMemcpyHostToDevice, stream));
            CK(cudaStreamSynchronize(stream));
            *dst = d;
        } else {
            Weight w;
            w.rows = (int)rows;
            w.cols = (int)cols;
            void* tmp = nullptr;
            CK(cudaMalloc(&tmp, need));
            CK(cudaMemcpyAsync(tmp, host, need, cudaMemcpyHostToDevice, stream));
            if (type == ACT_TYPE_Q8_0) {  // quants and scales apart; no f16 copy of the weight
                w.q = dalloc<uint8_t>(n);
                w.d = dalloc<f16>(n / 32);
                q8_0_split(static_cast<uint8_t*>(tmp), (int)rows, (int)cols, w.q, w.d, stream);
                wscratch_elems = std::max<long>(wscratch_elems, n);
            } else {
                w.h = dalloc<f16>(n);
                if (type == ACT_TYPE_F32) f32_to_f16(static_cast<float*>(tmp), w.h, n, stream);
                else CK(cudaMemcpyAsync(w.h, tmp, need, cudaMemcpyDeviceToDevice, stream));
            }
            CK(cudaStreamSynchronize(stream));
            CK(cudaFree(tmp));
            *wdst = w;
        }
        if (proj) {
            proj->bound = true;
            if (dora_proj) {  // lora_row_norm_sq, src/ac/lora.h:11-32
                proj->base = dalloc<float>(rows);
                std::vector<float> nsq(rows);
                for (long o = 0; o < rows; ++o) {
                    double s = (double)cols * 1e-12;
                    for (long i = 0; i < cols; ++i) {
                        const float v = f32[o * cols + i];
                        if (!std::isfinite(v)) throw Error(ACT_ERR_INVALID, "nonfinite DoRA base weight");
                        s += (double)v * v;
                    }
                    nsq[o] = (float)s;
                }
                CK(cudaMemcpyAsync(proj->base, nsq.data(), rows * 4, cudaMemcpyHostToDevice, stream));
                CK(cudaStreamSynchronize(stream));
                host_nsq[proj] = std::move(nsq);
            }
        }
        bound[name] = true;
    }

    std::map<Proj*, std::vector<float>> host_nsq;

    static float half_to_float(uint16_t h) {
        const uint32_t sign = (uint32_t)(h >> 15) << 31;
        uint32_t e = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
        if (e == 0) {
            if (man == 0) bits = sign;
            else {
                int k = -1;
                do { ++k; man <<= 1; } while (!(man & 0x400));
                man &= 0x3ff;
                bits = sign | (uint32_t)(127 - 15 - k) << 23 | man << 13;
            }
        } else if (e == 31) bits = sign | 0x7f800000u | man << 13;
        else bits = sign | (e + 112) << 23 | man << 13;
        float f;
        std::memcpy(&f, &bits, 4);
        return f;
    }

    void finalize() {
        if (finalized) throw Error(ACT_ERR_STATE, "already finalized");
        // completeness
        std::vector<std::string> missing;
        auto need = [&](const std::string& n) { if (!bound.count(n)) missing.push_back(n); };
        const std::string pre = mf ? "dit." : "lm.";
        for (int l = 0; l < L; ++l) {
            for (const char* nn : {"norm1", "norm_cross", "norm2"}) {
                need(pre + std::to_string(l) + "." + nn + ".weight");
                need(pre + std::to_string(l) + "." + nn + ".bias");
            }
            for (int t = 0; t < 7; ++t) need(pre + std::to_string(l) + "." + kTargets[t] + ".weight");
        }
        need(pre + "out_norm.weight");
        need(pre + "out_norm.bias");
        if (mf) {
            for (const char* nn : {"in_proj.weight", "out_proj.weight", "time_embed.0.weight", "time_embed.2.weight",
                                   "cond_proj.weight", "cond_proj.bias", "rope_freq_factors"})
                need(pre + nn);
            for (int i = 0; i < md.n_skip; ++i) need(pre + "skip." + std::to_string(i) + ".weight");
        } else {
            for (int q = 0; q < md.n_q; ++q) {
                need(pre + "emb." + std::to_string(q) + ".weight");
                need(pre + "head." + std::to_string(q) + ".weight");
            }
        }
        if (!missing.empty()) {
            std::string m = "missing tensors:";
            for (size_t i = 0; i < missing.size() && i < 8; ++i) m += " " + missing[i];
            throw Error(ACT_ERR_INVALID, m);
        }
        // parameters, reference order (src/mf/train.h:68-104)
        const float s = ad.alpha / (float)ad.rank;
        const bool dora = ad.type == ACT_ADAPTER_DORA_ROWS;
        int64_t off = 0;
        std::vector<CopyJob> jobs;
        for (int l = ad.first_layer; l < L; ++l)
            for (int t = 0; t < 7; ++t) {
                if (!(ad.targets >> t & 1)) continue;
                Proj& p = layers[l].p[t];
                p.adapted = true;
                p.dora = dora;
                p.r = ad.rank;
                p.RP = RP;
                p.s = s;
                const std::string stem = pre + std::to_string(l) + "." + kTargets[t] + ".weight";
                p.offA = off;
                ptable.push_back({stem + ".lora_A", off, p.r, p.in});
                off += (int64_t)p.r * p.in;
                p.offB = off;
                ptable.push_back({stem + ".lora_B", off, p.out, p.r});
                off += (int64_t)p.out * p.r;
                if (dora) {
                    p.offM = off;
                    ptable.push_back({stem + ".magnitude", off, 1, p.out});
                    off += p.out;
                }
            }
        nparam = off;
        layer_params.assign(L, {0, 0});
        for (const auto& pi : ptable) {
            const int l = std::atoi(pi.name.c_str() + pre.size());
            auto& r = layer_params[l];
            if (r.second == 0) r.first = pi.off;
            r.second = pi.off + pi.rows * pi.cols;
        }
        value = dalloc<float>(nparam);
        mom1 = dalloc<float>(nparam);
        mom2 = dalloc<float>(nparam);
        grad = dalloc<float>(nparam);
        decay = dalloc<uint8_t>(nparam);
        partials = dalloc<double>(1024);
        nonfinite_dev = dalloc<int>(1);
        {
            std::vector<uint8_t> dm(nparam, 0);
            std::vector<float> init(nparam, 0.f);
            std::mt19937 rng(ad.seed);
            std::normal_distribution<float> normal(0, 0.02f);
            for (auto& pi : ptable) {
                const bool isA = pi.name.size() > 7 && pi.name.compare(pi.name.size() - 7, 7, ".lora_A") == 0;
                const bool isB = pi.name.size() > 7 && pi.name.compare(pi.name.size() - 7, 7, ".lora_B") == 0;
                if (isA || isB) std::fill(dm.begin() + pi.off, dm.begin() + pi.off + pi.rows * pi.cols, 1);
                if (isA)
                    for (int64_t i = 0; i < pi.rows * pi.cols; ++i) init[pi.off + i] = normal(rng);
            }
            for (auto& lay : layers)
                for (auto& p : lay.p)
                    if (p.dora) {
                        const auto& nsq = host_nsq.at(&p);
                        for (int o = 0; o < p.out; ++o) init[p.offM + o] = std::sqrt(nsq[o]);
                    }
            CK(cudaMemcpyAsync(decay, dm.data(), nparam, cudaMemcpyHostToDevice, stream));
            CK(cudaMemcpyAsync(value, init.data(), nparam * 4, cudaMemcpyHostToDevice, stream));
            CK(cudaStreamSynchronize(stream));
        }
        // adapter working copies and DoRA scratch
        for (auto& lay : layers)
            for (auto& p : lay.p) {
                if (!p.adapted) continue;
                p.A_h = dalloc<f16>((size_t)RP * p.in);
                p.B_h = dalloc<f16>((size_t)p.out * RP);
                jobs.push_back({value + p.offA, p.A_h, p.r, p.in, p.in});
                jobs.push_back({value + p.offB, p.B_h, p.out, p.r, RP});
                max_job = std::max(max_job, std::max(p.r * p.in, p.out * p.r));
                if (p.dora) {
                    p.P = dalloc<float>((size_t)p.out * RP);
                    p.G = dalloc<float>((size_t)p.r * p.r);
                    p.Q = dalloc<float>((size_t)p.out * p.r);
                    p.nsq = dalloc<float>(p.out);
                    p.g = dalloc<float>(p.out);
                    p.dg = dalloc<float>(p.out);
                    p.scr = dalloc<float>((size_t)p.out + p.r * p.r);
                    p.colpart = dalloc<float>((size_t)DORA_COLSUM_PARTS * p.out);
                    p.colcnt = dalloc<int>((size_t)(p.out + 255) / 256);
                    p.BD = dalloc<f16>((size_t)p.out * RP);
                }
            }
        {
            std::vector<DoraJob> dj;
            dora_layer.assign(layers.size(), DoraSpan());
            for (size_t l = 0; l < layers.size(); ++l) {
                DoraSpan& sp = dora_layer[l];
                sp.first = (int)dj.size();
                for (auto& p : layers[l].p) {
                    if (!p.dora) continue;
                    DoraJob j;
                    j.A = value + p.offA; j.B = value + p.offB; j.m = value + p.offM;
                    j.P = p.P; j.base = p.base; j.G = p.G; j.Q = p.Q; j.nsq = p.nsq; j.g = p.g; j.dg = p.dg;
                    j.scr = p.scr; j.gm = grad + p.offM; j.gB = grad + p.offB; j.gA = grad + p.offA; j.BD = p.BD;
                    j.r = p.r; j.RP = p.RP; j.in = p.in; j.out = p.out; j.s = p.s;
                    dj.push_back(j);
                    sp.max_out = std::max(sp.max_out, p.out);
                    sp.max_in = std::max(sp.max_in, p.in);
                }
                sp.n = (int)dj.size() - sp.first;
                dora_max_out = std::max(dora_max_out, sp.max_out);
            }
            dora_n = (int)dj.size();
            if (dora_n) {
                CK(cudaStreamCreateWithFlags(&dora_stream, cudaStreamNonBlocking));
                CK(cudaEventCreateWithFlags(&ev_dora_fork, cudaEventDisableTiming));
                ev_dora.assign(layers.size(), nullptr);
                for (auto& e : ev_dora) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
                dora_async_ok = true;
                for (auto& lay : layers)
                    for (auto& p : lay.p) {
                        if (!p.dora) continue;
                        SkinnyArgs k;
                        k.M = p.out; k.K = p.in; k.nb = p.RP;
                        set_rank_weight(k, p.W, false);
                        k.B = p.A_h; k.ldb = p.in; k.kind = SKINNY_ACC; k.out = p.P; k.ldo = p.RP;
                        if (!skinny_supported(k)) dora_async_ok = false;
                    }
                dora_jobs_dev = dalloc<DoraJob>(dora_n);
                CK(cudaMemcpyAsync(dora_jobs_dev, dj.data(), sizeof(DoraJob) * dora_n, cudaMemcpyHostToDevice, stream));
                CK(cudaStreamSynchronize(stream));
            }
        }
        njobs = (int)jobs.size();
        jobs_dev = dalloc<CopyJob>(std::max(njobs, 1));
        if (njobs) CK(cudaMemcpyAsync(jobs_dev, jobs.data(), sizeof(CopyJob) * njobs, cudaMemcpyHostToDevice, stream));
        // rope table (src/ac/transformer.h:55-61 with freq_base 1): theta = pos / ff[i]
        if (mf) {
            if ((int)rope_ff.size() != md.head_dim / 2) throw Error(ACT_ERR_INVALID, "rope_freq_factors size mismatch");
            std::vector<float> tab((size_t)T * 64);
            for (int p = 0; p < T; ++p)
                for (int i = 0; i < 32; ++i) {
                    const float theta = (float)p / rope_ff[i];
                    tab[((size_t)p * 32 + i) * 2] = std::cos(theta);
                    tab[((size_t)p * 32 + i) * 2 + 1] = std::sin(theta);
                }
            rope = dalloc<float>(tab.size());
            CK(cudaMemcpyAsync(rope, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, stream));
            CK(cudaStreamSynchronize(stream));
        } else {
            // sin_positions (src/mg/lm.h:102-116), double phase
            std::vector<float> tab((size_t)T * D);
            const int half = D / 2;
            for (int t = 0; t < T; ++t)
                for (int i = 0; i < half; ++i) {
                    const double ph = (double)t / std::pow((double)md.max_period, (double)i / (double)md.pos_denominator);
                    tab[(size_t)t * D + i] = (float)std::cos(ph);
                    tab[(size_t)t * D + half + i] = (float)std::sin(ph);
                }
            pos = dalloc<float>(tab.size());
            CK(cudaMemcpyAsync(pos, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, stream));
            emb_dev = dalloc<float*>(md.n_q);
            CK(cudaMemcpyAsync(emb_dev, emb.data(), sizeof(float*) * md.n_q, cudaMemcpyHostToDevice, stream));
            CK(cudaStreamSynchronize(stream));
        }
        allocate_activations();
        if (wscratch_elems > 0)
            for (auto& slots : wscratch)
                for (auto& w : slots) w = dalloc<f16>(wscratch_elems);
        finalized = true;
    }

    void allocate_activations() {
        const long Mr = M, Cr = MC;
        for (int l = 0; l < L; ++l) {
            Layer& y = layers[l];
            if (l == 0) y.xin = x0f = dalloc<float>(Mr * D);
            else if (y.consumes) y.xin = dalloc<float>(Mr * D);
            else y.xin = layers[l - 1].xout;
            y.xmid = dalloc<float>(Mr * D);
            y.xmid2 = dalloc<float>(Mr * D);
            y.xout = dalloc<float>(Mr * D);
            for (int i = 0; i < 3; ++i) {
                y.mu[i] = dalloc<float>(Mr);
                y.rs[i] = dalloc<float>(Mr);
            }
            y.h1 = dalloc<f16>(Mr * D);
            y.hc = dalloc<f16>(Mr * D);
            y.f = dalloc<f16>(Mr * D);
            y.qkv = dalloc<f16>(Mr * 3 * D);
            y.o1 = dalloc<f16>(Mr * D);
            y.cq = dalloc<f16>(Mr * D);
            y.ckv = dalloc<f16>(Cr * 2 * D);
            y.o2 = dalloc<f16>(Mr * D);
            y.z = dalloc<f16>(Mr * F);
            y.gact = dalloc<f16>(Mr * F);
            y.lse1 = dalloc<float>((long)B * H * T);
            y.lse2 = dalloc<float>((long)B * H * T);
            for (int t = 0; t < 7; ++t) {
                if (!y.p[t].adapted) continue;
                y.U[t] = dalloc<f16>((t == 3 ? Cr : Mr) * RP);
                if (y.p[t].dora && (t == 0 || t == 1 || t == 4 || t == 6)) y.Yaux[t] = dalloc<f16>(Mr * y.p[t].out);
            }
            if (y.produces) {
                y.xsave_h = dalloc<f16>(Mr * D);
                y.dsaved = dalloc<float>(Mr * D);
            }
        }
        if (!x0f) x0f = layers[0].xin;
        const int lat = mf ? md.latent_dim : 8;
        x0 = dalloc<f16>(Mr * lat);
        vstar = dalloc<float>(Mr * lat);
        te1 = dalloc<float>((long)B * D);
        te = dalloc<float>((long)B * D);
        if (mf) hidden_h = dalloc<f16>(Cr * md.cond_dim);
        ctx_h = dalloc<f16>(Cr * D);
        xo = dalloc<f16>(Mr * D);
        muo = dalloc<float>(Mr);
        rso = dalloc<float>(Mr);
        outp = dalloc<float>(Mr * lat);
        dout = dalloc<f16>(Mr * lat);
        xprev_h = dalloc<f16>(Mr * D);
        dx = dalloc<float>(Mr * D);
        dtmp = dalloc<float>(Mr * D);
        dq_acc = dalloc<float>(Mr * D);
        dq_turn = dalloc<int>((size_t)B * H * ((T + 127) / 128));
        dvec = dalloc<float>((long)B * H * T);
        dxh = dalloc<f16>(Mr * D);
        dz = dalloc<f16>(Mr * F);
        dU = dalloc<f16>(std::max(Mr, Cr) * RP);
        dU_cond = dalloc<f16>(Cr * RP);
        dob = dalloc<f16>(Mr * D);
        dqkv = dalloc<f16>(Mr * 3 * D);
        dcq = dalloc<f16>(Mr * D);
        dckv = dalloc<f16>(Cr * 2 * D);
        cross_qsplit = ((T + 63) / 64 + 1) / 2;  // two query blocks per CTA
        dkv_acc = dalloc<float>((size_t)cross_qsplit * Cr * 2 * D);
        d_loss = dalloc<float>(B);
        loss_part = dalloc<float>((long)B * 32);
        h_loss = halloc<float>(B);
        if (mf) {
            const size_t nx = (size_t)B * md.latent_dim * T;
            h_clean = halloc<float>(nx); h_noise = halloc<float>(nx);
            h_hidden = halloc<float>((size_t)Cr * md.cond_dim);
            h_t = halloc<float>(B); h_tfeat = halloc<float>((size_t)B * md.time_dim); h_nvalid = halloc<int32_t>(B);
            h_start = halloc<float>(B);
            d_clean = dalloc<float>(nx); d_noise = dalloc<float>(nx);
            d_hidden = dalloc<float>((size_t)Cr * md.cond_dim);
            d_t = dalloc<float>(B); d_tfeat = dalloc<float>((size_t)B * md.time_dim); d_nvalid = dalloc<int32_t>(B);
            d_start = dalloc<float>(B);
        } else {
            const int sel = ad.frames - ad.prefix_frames;
            h_ids = halloc<int32_t>((size_t)B * md.n_q * T);
            h_tgt = halloc<int32_t>((size_t)B * md.n_q * sel);
            h_ctx = halloc<float>((size_t)Cr * D);
            d_ids = dalloc<int32_t>((size_t)B * md.n_q * T);
            d_tgt = dalloc<int32_t>((size_t)B * md.n_q * sel);
            mg_rowloss = dalloc<float>((size_t)B * std::max(sel, 1));
            d_ctx = dalloc<float>((size_t)Cr * D);
            if (C != Ctok) {
                d_mgvalid = dalloc<int32_t>(B);
                std::vector<int32_t> v((size_t)B, Ctok);
                CK(cudaMemcpy(d_mgvalid, v.data(), (size_t)B * 4, cudaMemcpyHostToDevice));
            }
            logits = dalloc<float>((size_t)B * md.n_q * T * md.card);   // [n_q][B][T][card]
            dlogits = dalloc<f16>((size_t)B * md.n_q * T * md.card);
        }
        CK(cudaStreamSynchronize(stream));
    }

    void optimizer(const act_opt* o, int* nonfinite) {
        if (!finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        if (!o || o->step <= 0 || !std::isfinite(o->lr) || o->lr <= 0 || !std::isfinite(o->clip) || o->clip <= 0 ||
            !(o->beta1 >= 0 && o->beta1 < 1) || !(o->beta2 >= 0 && o->beta2 < 1) || !(o->eps > 0) ||
            !(o->weight_decay >= 0))
            throw Error(ACT_ERR_INVALID, "invalid optimizer settings");
        const int count = o->count > 0 ? o->count : (count_override > 0 ? count_override : accumulated);
        if (count <= 0) throw Error(ACT_ERR_STATE, "empty gradient accumulation");
        const float bc1 = 1 - std::pow(o->beta1, (float)o->step), bc2 = 1 - std::pow(o->beta2, (float)o->step);
        CK(cudaMemsetAsync(nonfinite_dev, 0, sizeof(int), stream));
        timed(2, 0, 28.0 * nparam, [&] {
            adamw(value, mom1, mom2, grad, decay, nparam, (float)count, o->clip, o->lr, o->beta1, o->beta2, o->eps,
                  o->weight_decay, bc1, bc2, partials, nonfinite_dev, stream);
        });
        int bad = 0;
        CK(cudaMemcpyAsync(&bad, nonfinite_dev, sizeof(int), cudaMemcpyDeviceToHost, stream));
        check_kernel_error();
        collect_stats();
        accumulated = 0;
        count_override = 0;
        if (nonfinite) *nonfinite = bad;
        if (bad) throw Error(ACT_ERR_NONFINITE, "nonfinite optimizer update");
    }

    double step_flops(int n) const {
        // algorithmic FLOPs: 2 per multiply-add, no recompute, no padding.
        const double Td = T, Cd = C;
        double fwd = 0, bwd = 0;
        const double proj_tok = 2.0 * (3.0 * D * D + D * (double)D + D * (double)D + D * (double)D + 2.0 * D * F);
        for (int l = 0; l < L; ++l) {
            const bool grad_layer = l >= ad.first_layer;
            fwd += Td * proj_tok + 2.0 * Cd * D * 2.0 * D;
            fwd += attn_flops(1, T, true) + attn_flops(1, C, false);
            if (layers[l].consumes) fwd += 2.0 * Td * 2.0 * D * D;
            if (grad_layer) {
                bwd += Td * proj_tok;  // dX of every token projection
                if (l == ad.first_layer) bwd -= Td * 2.0 * 3.0 * D * D;  // no dX below the first adapted layer
                bwd += 2.0 * (attn_flops(1, T, true) + attn_flops(1, C, false));
                if (layers[l].consumes && l > ad.first_layer) bwd += 2.0 * Td * 2.0 * D * D;
                for (int t = 0; t < 7; ++t) {
                    const Proj& p = layers[l].p[t];
                    if (!p.adapted) continue;
                    const double rows = t == 3 ? Cd : Td;
                    fwd += rows * 2.0 * p.r * (p.in + p.out);
                    bwd += rows * 4.0 * p.r * (p.in + p.out);
                }
            }
        }
        if (mf) {
            fwd += 2.0 * Td * md.latent_dim * D * 2.0 + 2.0 * Cd * md.cond_dim * D;
            bwd += 2.0 * Td * md.latent_dim * D;
        } else {
            const double sel = (double)md.n_q * (ad.frames - ad.prefix_frames);
            fwd += 2.0 * sel * D * md.card;
            bwd += 2.0 * sel * D * md.card;
        }
        return n * (fwd + bwd);
    }

    void destroy() {
        if (stream) cudaStreamSynchronize(stream);
        for (auto& g : graphs) cudaGraphExecDestroy(g.second);
        graphs.clear();
        for (auto e : evpool) cudaEventDestroy(e);
        if (comm) ncclCommDestroy(comm);
        for (void* p : dallocs) cudaFree(p);
        for (void* p : hallocs) cudaFreeHost(p);
        if (side) cudaStreamSynchronize(side);
        if (dora_stream) cudaStreamSynchronize(dora_stream);
        if (comm_stream) cudaStreamSynchronize(comm_stream);
        if (ev_comm_fork) cudaEventDestroy(ev_comm_fork);
        if (ev_comm_join) cudaEventDestroy(ev_comm_join);
        if (comm_stream) cudaStreamDestroy(comm_stream);
        if (ev_fork) cudaEventDestroy(ev_fork);
        if (ev_join) cudaEventDestroy(ev_join);
        if (side) cudaStreamDestroy(side);
        for (auto e : ev_dora) if (e) cudaEventDestroy(e);
        if (ev_dora_fork) cudaEventDestroy(ev_dora_fork);
        if (dora_stream) cudaStreamDestroy(dora_stream);
        if (stream) cudaStreamDestroy(stream);
    }
};

// ------------------------------------------------------------------------------------------
// C ABI

namespace {

template <class Fn>
int guarded(act_ctx* ctx, Fn&& fn) {
    try {
        if (ctx) CK(cudaSetDevice(ctx->device));
        fn();
        return ACT_OK;
    } catch (const Error& e) {
        (ctx ? ctx->err : g_error) = e.what();
        return e.code;
    } catch (const std::exception& e) {
        (ctx ? ctx->err : g_error) = e.what();
        return ACT_ERR_INVALID;
    }
}

}  // namespace

extern "C" {

int act_create(act_ctx** out, int device, const act_model_desc* model, const act_adapter_desc* adapter) {
    if (!out || !model || !adapter) {
        g_error = "null argument";
        return ACT_ERR_INVALID;
    }
    *out = nullptr;
    auto* ctx = new act_ctx();
    try {
        ctx->setup(device, model, adapter);
        if (ctx->mf) ctx->skip.assign(model->n_skip, Weight());
        else {
            ctx->emb.assign(model->n_q, nullptr);
            ctx->head.assign(model->n_q, Weight());
        }
    } catch (const Error& e) {
        g_error = e.what();
        ctx->destroy();
        delete ctx;
        return e.code;
    } catch (const std::exception& e) {
        g_error = e.what();
        ctx->destroy();
        delete ctx;
        return ACT_ERR_INVALID;
    }
    *out = ctx;
    return ACT_OK;
}

int act_bind_weight(act_ctx* ctx, const char* name, int ggml_type, const void* host, size_t bytes) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] { ctx->bind(name, ggml_type, host, bytes); });
}

int act_finalize(act_ctx* ctx) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] { ctx->finalize(); });
}

int64_t act_param_count(act_ctx* ctx) { return ctx && ctx->finalized ? ctx->nparam : -1; }

int act_param_tensor_count(act_ctx* ctx) { return ctx && ctx->finalized ? (int)ctx->ptable.size() : -1; }

int act_param_tensor(act_ctx* ctx, int index, char* name, size_t cap, int64_t* offset, int64_t* rows, int64_t* cols) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        if (index < 0 || index >= (int)ctx->ptable.size()) throw Error(ACT_ERR_INVALID, "parameter index out of range");
        const auto& p = ctx->ptable[index];
        if (name && cap) {
            std::strncpy(name, p.name.c_str(), cap - 1);
            name[cap - 1] = 0;
        }
        if (offset) *offset = p.off;
        if (rows) *rows = p.rows;
        if (cols) *cols = p.cols;
    });
}

int act_set_params(act_ctx* ctx, const float* v, size_t n) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        if (!v || (int64_t)n != ctx->nparam) throw Error(ACT_ERR_INVALID, "parameter count mismatch");
        for (size_t i = 0; i < n; ++i)
            if (!std::isfinite(v[i])) throw Error(ACT_ERR_INVALID, "nonfinite adapter tensor");
        CK(cudaMemcpyAsync(ctx->value, v, n * 4, cudaMemcpyHostToDevice, ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
    });
}

int act_get_params(act_ctx* ctx, float* v, float* m, float* vv, size_t n) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        if ((int64_t)n != ctx->nparam) throw Error(ACT_ERR_INVALID, "parameter count mismatch");
        if (v) CK(cudaMemcpyAsync(v, ctx->value, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
        if (m) CK(cudaMemcpyAsync(m, ctx->mom1, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
        if (vv) CK(cudaMemcpyAsync(vv, ctx->mom2, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
    });
}

int act_set_moments(act_ctx* ctx, const float* m, const float* v, size_t n) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        if ((int64_t)n != ctx->nparam || !m || !v) throw Error(ACT_ERR_INVALID, "parameter count mismatch");
        CK(cudaMemcpyAsync(ctx->mom1, m, n * 4, cudaMemcpyHostToDevice, ctx->stream));
        CK(cudaMemcpyAsync(ctx->mom2, v, n * 4, cudaMemcpyHostToDevice, ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
    });
}

int act_get_grads(act_ctx* ctx, float* g, size_t n) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        if (!g || (int64_t)n != ctx->nparam) throw Error(ACT_ERR_INVALID, "parameter count mismatch");
        CK(cudaMemcpyAsync(g, ctx->grad, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
    });
}

int act_zero_grads(act_ctx* ctx) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        CK(cudaMemsetAsync(ctx->grad, 0, ctx->nparam * 4, ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
        ctx->accumulated = 0;
        ctx->count_override = 0;
    });
}

int act_mf_stage(act_ctx* ctx, const act_mf_batch* b) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        ctx->stage_mf(b);
    });
}

int act_mg_stage(act_ctx* ctx, const act_mg_batch* b) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        ctx->stage_mg(b);
    });
}

int act_run_staged(act_ctx* ctx, float* loss) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] { ctx->run_staged(loss); });
}

int act_mf_step(act_ctx* ctx, const act_mf_batch* b, float* loss) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        ctx->stage_mf(b);
        ctx->run_staged(loss);
    });
}

int act_mg_step(act_ctx* ctx, const act_mg_batch* b, float* loss) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        ctx->stage_mg(b);
        ctx->run_staged(loss);
    });
}

int act_nccl_get_unique_id(void* id) {
    if (!id) return ACT_ERR_INVALID;
    try {
        ncclUniqueId u;
        NK(ncclGetUniqueId(&u));
        std::memcpy(id, &u, sizeof(u));
        return ACT_OK;
    } catch (const Error& e) {
        g_error = e.what();
        return e.code;
    }
}

int act_nccl_init(act_ctx* ctx, const void* id, int nranks, int rank) {
    if (!ctx || !id) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (ctx->comm) throw Error(ACT_ERR_STATE, "communicator already initialised");
        if (nranks <= 0 || rank < 0 || rank >= nranks) throw Error(ACT_ERR_INVALID, "invalid rank or rank count");
        ncclUniqueId u;
        std::memcpy(&u, id, sizeof(u));
        // non-blocking: a peer that never joins ends in ncclCommAbort after the context's timeout
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        const ncclResult_t r = ncclCommInitRankConfig(&ctx->comm, nranks, u, rank, &cfg);
        if (r != ncclSuccess && r != ncclInProgress) {
            if (ctx->comm) ncclCommAbort(ctx->comm);
            ctx->comm = nullptr;
            throw Error(ACT_ERR_NCCL, std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
        }
        ctx->wait_nccl("communicator initialisation");
    });
}

int act_allreduce_grads(act_ctx* ctx, void* comm, int global_count) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->finalized) throw Error(ACT_ERR_STATE, "act_finalize has not been called");
        ncclComm_t c = comm ? static_cast<ncclComm_t>(comm) : ctx->comm;
        if (!c) throw Error(ACT_ERR_STATE, "no NCCL communicator");
        if (global_count <= 0) throw Error(ACT_ERR_INVALID, "invalid global sample count");
        ctx->timed(2, 0, 8.0 * ctx->nparam, [&] {
            const ncclResult_t r = ncclAllReduce(ctx->grad, ctx->grad, ctx->nparam, ncclFloat, ncclSum, c, ctx->stream);
            if (c == ctx->comm) ctx->nccl_call(r, "gradient all-reduce");
            else if (r != ncclSuccess) throw Error(ACT_ERR_NCCL, std::string("ncclAllReduce: ") + ncclGetErrorString(r));
        });
        ctx->count_override = global_count;
    });
}

int act_set_timeout(act_ctx* ctx, int64_t timeout_ms) {
    if (!ctx || timeout_ms < 0) return ACT_ERR_INVALID;
    ctx->timeout_ms = timeout_ms;
    return ACT_OK;
}

int act_set_deterministic(act_ctx* ctx, int enable) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        const bool on = enable != 0;
        if (on == ctx->deterministic) return;
        CK(cudaStreamSynchronize(ctx->stream));
        for (auto& g : ctx->graphs) cudaGraphExecDestroy(g.second);  // captured with the other order
        ctx->graphs.clear();
        ctx->deterministic = on;
    });
}

int act_set_grad_sync(act_ctx* ctx, int global_count) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (global_count < 0) throw Error(ACT_ERR_INVALID, "invalid global sample count");
        if (global_count > 0 && !ctx->comm) throw Error(ACT_ERR_STATE, "no NCCL communicator");
        ctx->grad_sync = global_count;
    });
}

int act_optimizer(act_ctx* ctx, const act_opt* o, int* nonfinite) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] { ctx->optimizer(o, nonfinite); });
}

const char* act_last_error(act_ctx* ctx) { return ctx ? ctx->err.c_str() : g_error.c_str(); }

void act_destroy(act_ctx* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    ctx->destroy();
    delete ctx;
}

void* act_stream(act_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int act_set_profiling(act_ctx* ctx, int enable) {
    if (!ctx) return ACT_ERR_INVALID;
    ctx->profiling = enable != 0;
    return ACT_OK;
}

int act_kernel_stats(act_ctx* ctx, int cls, double* ms, double* flops, double* bytes, int64_t* launches) {
    if (!ctx || cls < 0 || cls > 2) return ACT_ERR_INVALID;
    if (ms) *ms = ctx->stats[cls].ms;
    if (flops) *flops = ctx->stats[cls].flops;
    if (bytes) *bytes = ctx->stats[cls].bytes;
    if (launches) *launches = ctx->stats[cls].launches;
    return ACT_OK;
}

int act_reset_kernel_stats(act_ctx* ctx) {
    if (!ctx) return ACT_ERR_INVALID;
    for (auto& s : ctx->stats) s = KStat();
    return ACT_OK;
}

double act_step_flops(act_ctx* ctx, int n) { return ctx && ctx->finalized ? ctx->step_flops(n) : -1.0; }

int act_gelu_f16(int device, const uint16_t* z, uint16_t* g, uint16_t* dg, int64_t n, int direct) {
    void *dz = nullptr, *dgo = nullptr, *ddg = nullptr;
    cudaStream_t st = nullptr;
    auto cleanup = [&] {
        if (st) cudaStreamSynchronize(st);
        cudaFree(dz); cudaFree(dgo); cudaFree(ddg);
        if (st) cudaStreamDestroy(st);
    };
    try {
        if (!z || !g || !dg || n <= 0) throw Error(ACT_ERR_INVALID, "invalid GELU arguments");
        CK(cudaSetDevice(device));
        CK(cudaStreamCreate(&st));
        const int64_t n8 = (n + 7) / 8 * 8;  // the step's pass works on 8 values per thread
        CK(cudaMalloc(&dz, n8 * 2));
        CK(cudaMalloc(&dgo, n8 * 2));
        CK(cudaMalloc(&ddg, n8 * 2));
        CK(cudaMemsetAsync(dz, 0, n8 * 2, st));
        CK(cudaMemcpyAsync(dz, z, n * 2, cudaMemcpyHostToDevice, st));
        if (direct) {
            gelu_check(static_cast<const uint16_t*>(dz), static_cast<uint16_t*>(dgo), static_cast<uint16_t*>(ddg), n,
                       st);
        } else {  // the training step's pass: gelu into dgo, gelu' over the input in place
            gelu_fwd(static_cast<f16*>(dz), static_cast<f16*>(dgo), n8, 1, st);
            CK(cudaMemcpyAsync(ddg, dz, n8 * 2, cudaMemcpyDeviceToDevice, st));
        }
        CK(cudaGetLastError());
        CK(cudaMemcpyAsync(g, dgo, n * 2, cudaMemcpyDeviceToHost, st));
        CK(cudaMemcpyAsync(dg, ddg, n * 2, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        cleanup();
        return ACT_OK;
    } catch (const Error& e) {
        g_error = e.what();
        cleanup();
        return e.code;
    } catch (const std::exception& e) {
        g_error = e.what();
        cleanup();
        return ACT_ERR_CUDA;
    }
}

// The rank-block kernel on host buffers: A as f16 bits, or (Aq8 non-null) as the Q8_0 blocks of
// the weight it is read from ([M][K] when a_mn is 0, [K][M] when 1), kept quantised on the device.
static int rank_gemm_host(int device, int kind, const void* A, const void* Aq8, const void* B, float* C, int M, int K,
                          int nb, int a_mn, int b_mn, float alpha, int splits, int reps, float* ms_per_call) {
    void *dA = nullptr, *dB = nullptr, *dC = nullptr, *dQ = nullptr, *dD = nullptr;
    int* derr = nullptr;
    cudaStream_t st = nullptr;
    auto cleanup = [&] {
        if (st) cudaStreamSynchronize(st);
        cudaFree(dA); cudaFree(dB); cudaFree(dC); cudaFree(derr); cudaFree(dQ); cudaFree(dD);
        if (st) cudaStreamDestroy(st);
    };
    try {
        if ((!A && !Aq8) || !B || !C || M <= 0 || K <= 0 || nb <= 0 || kind < 0 || kind > 2)
            throw Error(ACT_ERR_INVALID, "invalid rank-GEMM arguments");
        const int wrows = a_mn ? K : M, wcols = a_mn ? M : K;  // the stored matrix A is read from
        if (Aq8 && wcols % 32) throw Error(ACT_ERR_INVALID, "Q8_0 rows must be whole 32-blocks");
        CK(cudaSetDevice(device));
        CK(cudaStreamCreate(&st));
        const size_t cn = (size_t)M * nb;
        if (Aq8) {
            const size_t nblk = (size_t)wrows * wcols / 32;
            CK(cudaMalloc(&dA, nblk * 34));
            CK(cudaMalloc(&dQ, (size_t)wrows * wcols));
            CK(cudaMalloc(&dD, nblk * 2));
        } else {
            CK(cudaMalloc(&dA, (size_t)M * K * 2));
        }
        CK(cudaMalloc(&dB, (size_t)nb * K * 2));
        CK(cudaMalloc(&dC, cn * 4));
        CK(cudaMalloc(&derr, sizeof(int)));
        CK(cudaMemsetAsync(derr, 0, sizeof(int), st));
        if (Aq8) {
            CK(cudaMemcpyAsync(dA, Aq8, (size_t)wrows * wcols / 32 * 34, cudaMemcpyHostToDevice, st));
            q8_0_split(static_cast<const uint8_t*>(dA), wrows, wcols, static_cast<uint8_t*>(dQ),
                       static_cast<f16*>(dD), st);
        } else {
            CK(cudaMemcpyAsync(dA, A, (size_t)M * K * 2, cudaMemcpyHostToDevice, st));
        }
        CK(cudaMemcpyAsync(dB, B, (size_t)nb * K * 2, cudaMemcpyHostToDevice, st));
        SkinnyArgs g;
        g.M = M; g.K = K; g.nb = nb;
        g.lda = a_mn ? M : K; g.a_mn = a_mn != 0;
        if (Aq8) {
            g.Aq = static_cast<const uint8_t*>(dQ); g.Ad = static_cast<const f16*>(dD); g.ldad = wrows;
        } else {
            g.A = static_cast<const f16*>(dA);
        }
        g.B = static_cast<const f16*>(dB); g.ldb = b_mn ? nb : K; g.b_mn = b_mn != 0;
        g.kind = kind; g.alpha = alpha; g.out = dC; g.ldo = kind == SKINNY_ACC_T ? M : nb;
        g.splits = splits;
        if (kind == SKINNY_STORE) {
            CK(cudaMemsetAsync(dC, 0, cn * 4, st));
        } else {
            CK(cudaMemcpyAsync(dC, C, cn * 4, cudaMemcpyHostToDevice, st));
        }
        if (!skinny_supported(g)) throw Error(ACT_ERR_INVALID, "operands not supported by the rank-GEMM kernel");
        skinny_gemm(g, derr, st);
        CK(cudaGetLastError());
        if (reps > 0 && ms_per_call) {
            cudaGraph_t graph;
            cudaGraphExec_t exec;
            CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            for (int i = 0; i < reps; ++i) skinny_gemm(g, derr, st);
            CK(cudaStreamEndCapture(st, &graph));
            CK(cudaGraphInstantiate(&exec, graph, 0));
            CK(cudaGraphLaunch(exec, st));
            cudaEvent_t e0, e1;
            CK(cudaEventCreate(&e0));
            CK(cudaEventCreate(&e1));
            CK(cudaEventRecord(e0, st));
            CK(cudaGraphLaunch(exec, st));
            CK(cudaEventRecord(e1, st));
            CK(cudaEventSynchronize(e1));
            float ms = 0;
            CK(cudaEventElapsedTime(&ms, e0, e1));
            *ms_per_call = ms / reps;
            cudaEventDestroy(e0);
            cudaEventDestroy(e1);
            cudaGraphExecDestroy(exec);
            cudaGraphDestroy(graph);
        }
        if (kind == SKINNY_STORE) {
            std::vector<uint16_t> hb(cn);
            // the f16 result occupies the first cn * 2 bytes of dC (row stride nb)
            CK(cudaMemcpyAsync(hb.data(), dC, cn * 2, cudaMemcpyDeviceToHost, st));
            CK(cudaStreamSynchronize(st));
            for (size_t i = 0; i < cn; ++i) C[i] = act_ctx::half_to_float(hb[i]);
        } else {
            CK(cudaMemcpyAsync(C, dC, cn * 4, cudaMemcpyDeviceToHost, st));
        }
        int e = 0;
        CK(cudaMemcpyAsync(&e, derr, sizeof(int), cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        if (e) throw Error(ACT_ERR_CUDA, "rank-GEMM kernel reported a timed-out wait (code " + std::to_string(e) + ")");
        cleanup();
        return ACT_OK;
    } catch (const Error& e) {
        g_error = e.what();
        cleanup();
        return e.code;
    } catch (const std::exception& e) {
        g_error = e.what();
        cleanup();
        return ACT_ERR_CUDA;
    }
}

int act_rank_gemm_f16(int device, int kind, const void* A, const void* B, float* C, int M, int K, int nb, int a_mn,
                      int b_mn, float alpha, int splits, int reps, float* ms_per_call) {
    return rank_gemm_host(device, kind, A, nullptr, B, C, M, K, nb, a_mn, b_mn, alpha, splits, reps, ms_per_call);
}

int act_rank_gemm_q8_0(int device, int kind, const void* Aq8, const void* B, float* C, int M, int K, int nb, int a_mn,
                       int b_mn, float alpha, int splits, int reps, float* ms_per_call) {
    if (!Aq8) return ACT_ERR_INVALID;
    return rank_gemm_host(device, kind, nullptr, Aq8, B, C, M, K, nb, a_mn, b_mn, alpha, splits, reps, ms_per_call);
}

namespace {

// Stand-alone projection GEMM on host buffers: C[M][N] (fp32) = A[M][K] . B(n,k) with f16 A and
// B either f16 (B) or the Q8_0 blocks of the weight (Bq8: [N][K] or [K][N] as b_mn_major says).
int gemm_entry(int device, const void* A, const void* B, const void* Bq8, void* C, int M, int N, int K,
               int b_mn_major, int path, int reps, float* ms_per_call) {
    void *dA = nullptr, *dB = nullptr, *dC = nullptr, *dsk = nullptr, *dflag = nullptr, *dq = nullptr, *dd = nullptr;
    int* derr = nullptr;
    cudaStream_t st = nullptr;
    auto cleanup = [&] {
        if (st) cudaStreamSynchronize(st);
        cudaFree(dA); cudaFree(dB); cudaFree(dC); cudaFree(derr); cudaFree(dsk); cudaFree(dflag);
        cudaFree(dq); cudaFree(dd);
        if (st) cudaStreamDestroy(st);
    };
    try {
        if (!A || !(B || Bq8) || !C || M <= 0 || N <= 0 || K <= 0) throw Error(ACT_ERR_INVALID, "invalid GEMM arguments");
        const int wrows = b_mn_major ? K : N, wcols = b_mn_major ? N : K;  // the weight [out][in]
        if (Bq8 && (wcols % 32 || path == 1 || path == 2))
            throw Error(ACT_ERR_INVALID, "Q8_0 weights take the 2-CTA paths (0, 3, 4, 5) with whole blocks");
        CK(cudaSetDevice(device));
        CK(cudaStreamCreate(&st));
        CK(cudaMalloc(&dA, (size_t)M * K * 2));
        CK(cudaMalloc(&dC, (size_t)M * N * 4));
        CK(cudaMalloc(&derr, sizeof(int)));
        CK(cudaMemsetAsync(derr, 0, sizeof(int), st));
        CK(cudaMemcpyAsync(dA, A, (size_t)M * K * 2, cudaMemcpyHostToDevice, st));
        GemmArgs g;
        g.M = M; g.N = N; g.K1 = K;
        g.A1 = static_cast<const f16*>(dA); g.lda1 = K;
        g.b_kmajor = !b_mn_major;
        if (Bq8) {
            const size_t nb = (size_t)N * K / 32;
            CK(cudaMalloc(&dB, nb * 34));
            CK(cudaMalloc(&dq, (size_t)N * K));
            CK(cudaMalloc(&dd, nb * 2));
            CK(cudaMemcpyAsync(dB, Bq8, nb * 34, cudaMemcpyHostToDevice, st));
            q8_0_split(static_cast<const uint8_t*>(dB), wrows, wcols, static_cast<uint8_t*>(dq), static_cast<f16*>(dd), st);
            g.B1q = static_cast<const uint8_t*>(dq); g.ldb1 = wcols;
            g.B1d = static_cast<const f16*>(dd); g.ldd1 = wrows;
        } else {
            CK(cudaMalloc(&dB, (size_t)N * K * 2));
            CK(cudaMemcpyAsync(dB, B, (size_t)N * K * 2, cudaMemcpyHostToDevice, st));
            g.B1 = static_cast<const f16*>(dB); g.ldb1 = wcols;
        }
        g.mode = EPI_STORE_F32; g.out = dC; g.ldo = N;
        const bool tc = path >= 2 || (path == 0 && gemm_tc_supported(g));
        if (tc && !gemm_tc_supported(g)) throw Error(ACT_ERR_INVALID, "shape not supported by the tcgen05 path");
        if (path >= 3 && !gemm_tc2_supported(g))
            throw Error(ACT_ERR_INVALID, "shape not supported by the 2-CTA path");
        if (path < 0 || path > 5) throw Error(ACT_ERR_INVALID, "unknown GEMM path");
        if (path == 0 || path == 3) {
            int sms = 0;
            CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
            CK(cudaMalloc(&dsk, sizeof(float) * gemm_sk_part_floats(sms)));
            CK(cudaMalloc(&dflag, sizeof(int) * gemm_sk_flag_count(sms)));
            CK(cudaMemsetAsync(dflag, 0, sizeof(int) * gemm_sk_flag_count(sms), st));
            g.sk_part = static_cast<float*>(dsk);
            g.sk_flag = static_cast<int*>(dflag);
        }
        auto run = [&] {
            if (path == 3 || path == 5) gemm_tc2(g, derr, st);
            else if (path == 4) gemm_tc2_width(g, derr, st, 128);
            else if (path == 0 && tc) gemm_tc_auto(g, derr, st);
            else if (tc) gemm_tc(g, derr, st);
            else gemm(g, st);
        };
        run();
        CK(cudaGetLastError());
        if (reps > 0 && ms_per_call) {
            // time `reps` launches replayed from a CUDA graph: device time without host gaps
            cudaGraph_t graph;
            cudaGraphExec_t exec;
            CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            for (int i = 0; i < reps; ++i) run();
            CK(cudaStreamEndCapture(st, &graph));
            CK(cudaGraphInstantiate(&exec, graph, 0));
            CK(cudaGraphLaunch(exec, st));
            cudaEvent_t e0, e1;
            CK(cudaEventCreate(&e0));
            CK(cudaEventCreate(&e1));
            CK(cudaEventRecord(e0, st));
            CK(cudaGraphLaunch(exec, st));
            CK(cudaEventRecord(e1, st));
            CK(cudaEventSynchronize(e1));
            float ms = 0;
            CK(cudaEventElapsedTime(&ms, e0, e1));
            *ms_per_call = ms / reps;
            cudaEventDestroy(e0);
            cudaEventDestroy(e1);
            cudaGraphExecDestroy(exec);
            cudaGraphDestroy(graph);
        }
        CK(cudaMemcpyAsync(C, dC, (size_t)M * N * 4, cudaMemcpyDeviceToHost, st));
        int e = 0;
        CK(cudaMemcpyAsync(&e, derr, sizeof(int), cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        if (e) throw Error(ACT_ERR_CUDA, "GEMM kernel reported a timed-out wait (code " + std::to_string(e) + ")");
        cleanup();
        return ACT_OK;
    } catch (const Error& e) {
        g_error = e.what();
        cleanup();
        return e.code;
    } catch (const std::exception& e) {
        g_error = e.what();
        cleanup();
        return ACT_ERR_INVALID;
    }
}

}  // namespace

int act_gemm_f16(int device, const void* A, const void* B, void* C, int M, int N, int K, int b_mn_major, int path,
                 int reps, float* ms_per_call) {
    // path 0 auto, 1 mma.sync, 2 tcgen05, 3 2-CTA (stream-K where it pays), 4 2-CTA 128-wide,
    // 5 2-CTA whole tiles only
    return gemm_entry(device, A, B, nullptr, C, M, N, K, b_mn_major, path, reps, ms_per_call);
}

int act_gemm_q8_0(int device, const void* A, const void* Bq8, void* C, int M, int N, int K, int b_mn_major, int path,
                  int reps, float* ms_per_call) {
    return gemm_entry(device, A, nullptr, Bq8, C, M, N, K, b_mn_major, path, reps, ms_per_call);
}

int act_attention(int device, const void* q, const void* k, const void* v, const void* dout, int clips, int T,
                  int Tk, int H, const int32_t* nvalid, int causal, int zero_key, const float* rope, void* o,
                  float* lse, void* dq, void* dk, void* dv, float* ms_fwd, float* ms_bwd) {
    // Stand-alone attention forward + backward on host buffers (tests and the kernel sweep).
    std::vector<void*> bufs;
    cudaStream_t st = nullptr;
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    auto cleanup = [&] {
        if (st) cudaStreamSynchronize(st);
        for (void* b : bufs) cudaFree(b);
        for (auto e : ev)
            if (e) cudaEventDestroy(e);
        if (st) cudaStreamDestroy(st);
    };
    try {
        if (!q || !k || !v || !o || !lse || clips <= 0 || T <= 0 || Tk <= 0 || H <= 0)
            throw Error(ACT_ERR_INVALID, "invalid attention arguments");
        if (causal && Tk != T) throw Error(ACT_ERR_INVALID, "causal attention needs Tk == T");
        CK(cudaSetDevice(device));
        CK(cudaStreamCreate(&st));
        for (auto& e : ev) CK(cudaEventCreate(&e));
        const long D = (long)H * 64, rq = (long)clips * T, rk = (long)clips * Tk;
        auto up = [&](const void* h, size_t bytes) -> void* {
            void* d = nullptr;
            CK(cudaMalloc(&d, std::max<size_t>(bytes, 16)));
            bufs.push_back(d);
            if (h) CK(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, st));
            else CK(cudaMemsetAsync(d, 0, bytes, st));
            return d;
        };
        AttnArgs a;
        a.q = static_cast<const f16*>(up(q, rq * D * 2));
        a.k = static_cast<const f16*>(up(k, rk * D * 2));
        a.v = static_cast<const f16*>(up(v, rk * D * 2));
        a.ldq = a.ldk = a.ldv = D;
        a.T = T; a.Tk = Tk; a.H = H; a.clips = clips;
        a.nvalid = nvalid ? static_cast<const int*>(up(nvalid, clips * 4)) : nullptr;
        a.causal = causal; a.zero_key = zero_key;
        a.rope = rope ? static_cast<const float*>(up(rope, (size_t)T * 64 * 4)) : nullptr;
        a.rope_load = rope ? 1 : 0;  // unrotated inputs: rotate while staging
        if (rope && Tk > T) throw Error(ACT_ERR_INVALID, "RoPE needs Tk <= T");
        a.scale = 0.125f;
        a.o = static_cast<f16*>(up(nullptr, rq * D * 2));
        a.ldo = D;
        a.lse = static_cast<float*>(up(nullptr, rq * H * 4));
        int* derr = static_cast<int*>(up(nullptr, sizeof(int)));
        const bool mma_only = std::getenv("ACTRAIN_ATTN_MMA") != nullptr;
        const bool x_tc = xattn_tc_supported(a) && !mma_only;  // at most 64 keys, as cross-attention runs
        const bool tc_fwd = !x_tc && attn_fwd_tc_supported(a) && !mma_only;
        CK(cudaEventRecord(ev[0], st));
        if (x_tc) xattn_fwd_tc(a, derr, st);
        else if (tc_fwd) attn_fwd_tc(a, derr, st);
        else attn_fwd(a, st);
        CK(cudaEventRecord(ev[1], st));
        CK(cudaGetLastError());
        const bool bwd = dout && dq && dk && dv;
        f16* ddq = nullptr;
        if (bwd) {
            a.dout = static_cast<const f16*>(up(dout, rq * D * 2));
            a.lddo = D;
            a.dvec = static_cast<float*>(up(nullptr, rq * H * 4));
            a.dq_acc = static_cast<float*>(up(nullptr, rq * D * 4));
            a.ldq_acc = D;
            a.dk = static_cast<f16*>(up(nullptr, rk * D * 2));
            a.dv = static_cast<f16*>(up(nullptr, rk * D * 2));
            a.lddk = a.lddv = D;
            ddq = static_cast<f16*>(up(nullptr, rq * D * 2));
            if (x_tc) {  // dQ straight to f16, dK / dV through one fp32 slice per 128 queries
                a.dq_h = ddq;
                a.lddq_h = D;
                a.qsplit = (T + 127) / 128;
                a.dk_acc = static_cast<float*>(up(nullptr, (size_t)a.qsplit * rk * D * 4));
                a.dv_acc = static_cast<float*>(up(nullptr, (size_t)a.qsplit * rk * D * 4));
            }
            CK(cudaEventRecord(ev[2], st));
            if (x_tc) {
                xattn_bwd_tc(a, derr, st);
            } else if (attn_bwd_tc_supported(a) && !mma_only) {
                attn_bwd_tc(a, derr, st);
            } else if (Tk <= 64) {  // few keys: query-split backward, as the training step runs it
                a.qsplit = (T + 63) / 64;
                a.dk_acc = static_cast<float*>(up(nullptr, (size_t)a.qsplit * rk * D * 4));
                a.dv_acc = static_cast<float*>(up(nullptr, (size_t)a.qsplit * rk * D * 4));
                attn_bwd(a, st);
                attn_dkv_finish(a, st);
            } else {
                attn_bwd(a, st);
            }
            if (!x_tc) attn_dq_finish(a, ddq, D, nullptr, st);
            CK(cudaEventRecord(ev[3], st));
            CK(cudaGetLastError());
        }
        CK(cudaMemcpyAsync(o, a.o, rq * D * 2, cudaMemcpyDeviceToHost, st));
        CK(cudaMemcpyAsync(lse, a.lse, rq * H * 4, cudaMemcpyDeviceToHost, st));
        if (bwd) {
            CK(cudaMemcpyAsync(dq, ddq, rq * D * 2, cudaMemcpyDeviceToHost, st));
            CK(cudaMemcpyAsync(dk, a.dk, rk * D * 2, cudaMemcpyDeviceToHost, st));
            CK(cudaMemcpyAsync(dv, a.dv, rk * D * 2, cudaMemcpyDeviceToHost, st));
        }
        int e = 0;
        CK(cudaMemcpyAsync(&e, derr, sizeof(int), cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        if (e) throw Error(ACT_ERR_CUDA, "attention kernel reported a timed-out wait (code " + std::to_string(e) + ")");
        if (ms_fwd) CK(cudaEventElapsedTime(ms_fwd, ev[0], ev[1]));
        if (ms_bwd) {
            *ms_bwd = 0.f;
            if (bwd) CK(cudaEventElapsedTime(ms_bwd, ev[2], ev[3]));
        }
        cleanup();
        return ACT_OK;
    } catch (const Error& e) {
        g_error = e.what();
        cleanup();
        return e.code;
    } catch (const std::exception& e) {
        g_error = e.what();
        cleanup();
        return ACT_ERR_INVALID;
    }
}

int act_path_counts(act_ctx* ctx, int64_t* counts, int n) {
    if (!ctx || !counts || n < 0) return ACT_ERR_INVALID;
    for (int i = 0; i < n; ++i) counts[i] = i < ACT_PATH_COUNT ? ctx->path_count[i] : 0;
    return ACT_OK;
}

int act_wait_probe(act_ctx* ctx, int64_t limit_ns) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (limit_ns <= 0 || limit_ns > 10000000000LL) throw Error(ACT_ERR_INVALID, "wait limit out of range");
        wait_probe(ctx->probe_flag, limit_ns, ctx->kerr, ctx->stream);
        CK(cudaGetLastError());
        ctx->check_kernel_error();
    });
}

int act_mg_staged(act_ctx* ctx, int32_t* ids, size_t n_ids, int32_t* targets, size_t n_targets) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (ctx->mf) throw Error(ACT_ERR_INVALID, "not a MusicGen context");
        if (ctx->staged_n <= 0) throw Error(ACT_ERR_STATE, "no staged batch");
        const size_t n = ctx->staged_n, nq = ctx->md.n_q, sel = ctx->ad.frames - ctx->ad.prefix_frames;
        if (!ids || !targets || n_ids != n * nq * ctx->T || n_targets != n * nq * sel)
            throw Error(ACT_ERR_INVALID, "staged buffer size mismatch");
        CK(cudaMemcpyAsync(ids, ctx->d_ids, n_ids * 4, cudaMemcpyDeviceToHost, ctx->stream));
        CK(cudaMemcpyAsync(targets, ctx->d_tgt, n_targets * 4, cudaMemcpyDeviceToHost, ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
    });
}

int act_mf_staged(act_ctx* ctx, float* clean, float* noise, size_t n_values) {
    if (!ctx) return ACT_ERR_INVALID;
    return guarded(ctx, [&] {
        if (!ctx->mf) throw Error(ACT_ERR_INVALID, "not a MelodyFlow context");
        if (ctx->staged_n <= 0) throw Error(ACT_ERR_STATE, "no staged batch");
        const size_t nx = (size_t)ctx->staged_n * ctx->md.latent_dim * ctx->T;
        if (n_values < nx) throw Error(ACT_ERR_INVALID, "buffers too small");
        if (clean) CK(cudaMemcpyAsync(clean, ctx->d_clean, nx * 4, cudaMemcpyDeviceToHost, ctx->stream));
        if (noise) CK(cudaMemcpyAsync(noise, ctx->d_noise, nx * 4, cudaMemcpyDeviceToHost, ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
    });
}

int act_q8_0_dequant(int device, const void* blocks, int64_t nblocks, float* out_f32, uint16_t* out_f16) {
    void *db = nullptr, *df = nullptr, *dh = nullptr;
    cudaStream_t st = nullptr;
    auto cleanup = [&] {
        if (st) cudaStreamSynchronize(st);
        cudaFree(db); cudaFree(df); cudaFree(dh);
        if (st) cudaStreamDestroy(st);
    };
    try {
        if (!blocks || nblocks <= 0 || (!out_f32 && !out_f16)) throw Error(ACT_ERR_INVALID, "invalid Q8_0 arguments");
        CK(cudaSetDevice(device));
        CK(cudaStreamCreate(&st));
        const size_t n = (size_t)nblocks * 32;
        CK(cudaMalloc(&db, (size_t)nblocks * 34));
        CK(cudaMemcpyAsync(db, blocks, (size_t)nblocks * 34, cudaMemcpyHostToDevice, st));
        if (out_f32) {
            CK(cudaMalloc(&df, n * 4));
            q8_0_to_f32(static_cast<const uint8_t*>(db), nblocks, static_cast<float*>(df), st);
            CK(cudaMemcpyAsync(out_f32, df, n * 4, cudaMemcpyDeviceToHost, st));
        }
        if (out_f16) {
            CK(cudaMalloc(&dh, n * 2));
            q8_0_to_f16(static_cast<const uint8_t*>(db), nblocks, static_cast<f16*>(dh), st);
            CK(cudaMemcpyAsync(out_f16, dh, n * 2, cudaMemcpyDeviceToHost, st));
        }
        CK(cudaGetLastError());
        CK(cudaStreamSynchronize(st));
        cleanup();
        return ACT_OK;
    } catch (const Error& e) {
        g_error = e.what();
        cleanup();
        return e.code;
    } catch (const std::exception& e) {
        g_error = e.what();
        cleanup();
        return ACT_ERR_INVALID;
    }
}

int64_t act_graph_kernel_nodes(act_ctx* ctx, int n) {
    if (!ctx) return -1;
    auto it = ctx->kernel_nodes.find(n);
    return it == ctx->kernel_nodes.end() ? -1 : it->second;
}

}  // extern "C"
