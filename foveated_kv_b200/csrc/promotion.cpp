// Spike drain + promotion of exact fp16 rows into near-tier headroom.
//
// Host side of the closed loop of the reference's PromotionPipeline
// (csrc/promotion_pipeline.cpp:20-248): drain_spikes filters the fused
// kernel's per-head spike flags (GQA dedup, cooldown, position dedup, budget)
// and queues records; one worker std::thread per pipeline takes everything
// queued at once, packs the exact fp16 K/V rows of those records from the
// host archive (mmapped file or caller memory) into one pinned staging buffer
// together with their destination slots (near_valid[b, h], counted on a host
// shadow) and the new counts, moves the batch to the device with ONE
// cudaMemcpyAsync on its own stream, and launches a scatter kernel that writes
// the rows, then a second one that stores the counts.  Stream order makes a
// count visible only after the rows it covers, so a decode launch that reads
// near_valid sees either the old count or the new count with its rows in
// place.
//
// Differences from the reference, all identical at B = 1: near_valid is per
// (b, kv head) and GQA dedup / cooldown / position dedup are keyed by batch
// row too (the reference keys them by kv head and promotes batch 0 only,
// promotion_pipeline.cpp:117-139,230).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <thread>
#include <unordered_map>
#include <set>
#include <tuple>
#include <vector>

#include "fkv_common.h"

namespace {

struct Record {
    int layer, b, h, arc_local;
};

struct Archive {
    const uint16_t* k = nullptr;
    const uint16_t* v = nullptr;
    void* map_k = nullptr;
    void* map_v = nullptr;
    size_t map_bytes = 0;
    int B = 0, H = 0, S = 0, D = 0;
    std::vector<std::unordered_map<int32_t, int32_t>> pos_to_local;   // [b * H + h]
};

struct Blob {
    uint16_t* near_k = nullptr;
    uint16_t* near_v = nullptr;
    int32_t* near_valid = nullptr;
    int B = 0, H = 0, Np = 0, D = 0;
    std::vector<int32_t> shadow;   // host copy of near_valid; the worker is its only writer
};

constexpr int kStagingBufs = 2;   // pinned batch buffers in flight

}  // namespace

struct FkvPromo {
    int n_layers, cooldown, budget, device;
    std::vector<Archive> archives;
    std::vector<Blob> blobs;
    std::set<std::tuple<int, int, int, int32_t>> promoted;   // (layer, b, h, position)
    std::unordered_map<uint64_t, int> last_step;

    std::mutex mu;
    std::condition_variable cv, idle_cv;
    std::deque<Record> queue;
    bool busy = false;
    std::atomic<bool> running{true};
    std::thread worker;

    std::atomic<uint64_t> detected{0}, queued{0}, deduplicated{0}, cooled{0}, completed{0},
        headroom_full{0};

    // device resources, created by the worker on first use: its stream,
    // kStagingBufs pinned batch buffers (each reused once the copy out of it
    // has completed) and one device staging buffer (reused in stream order)
    bool cuda_ready = false;
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    uint8_t* staging[kStagingBufs] = {};
    size_t staging_bytes[kStagingBufs] = {};
    cudaEvent_t staging_ev[kStagingBufs] = {};
    int next_buf = 0;
    void* dev_stage = nullptr;
    size_t dev_stage_bytes = 0;
    std::string worker_error;

    ~FkvPromo();
    void run();
    bool ensure_cuda();
    void promote_batch(std::vector<Record>& batch);
    void promote_layer(int layer, const Record* recs, size_t n);
};

void FkvPromo::run() {
    while (true) {
        std::vector<Record> batch;
        {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return !queue.empty() || !running.load(); });
            if (queue.empty()) break;   // stopping and drained
            batch.assign(queue.begin(), queue.end());
            queue.clear();
            busy = true;
        }
        promote_batch(batch);
        {
            std::lock_guard<std::mutex> lk(mu);
            busy = false;
        }
        idle_cv.notify_all();
    }
    idle_cv.notify_all();
}

bool FkvPromo::ensure_cuda() {
    if (cuda_ready) return true;
    if (cudaSetDevice(device) != cudaSuccess) return false;
    if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess) return false;
    if (cudaEventCreateWithFlags(&done, cudaEventDisableTiming) != cudaSuccess) return false;
    for (auto& e : staging_ev)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return false;
    cuda_ready = true;
    return true;
}

void FkvPromo::promote_batch(std::vector<Record>& batch) {
    if (!ensure_cuda()) {
        worker_error = "promotion worker: CUDA setup failed";
        return;
    }
    // records of one layer share a near tier and an archive: one batch each
    std::stable_sort(batch.begin(), batch.end(),
                     [](const Record& a, const Record& b) { return a.layer < b.layer; });
    size_t i = 0;
    while (i < batch.size()) {
        size_t j = i;
        while (j < batch.size() && batch[j].layer == batch[i].layer) ++j;
        promote_layer(batch[i].layer, batch.data() + i, j - i);
        i = j;
    }
}

void FkvPromo::promote_layer(int layer, const Record* recs, size_t n) {
    Archive& a = archives[layer];
    Blob& bl = blobs[layer];
    if (!a.k || !bl.near_k) return;   // nothing to promote into (reference: :215-216)
    const int D = a.D;
    // destinations from the host shadow of near_valid; full headroom is counted
    std::vector<const Record*> ok;
    std::vector<int64_t> dst;
    std::vector<int32_t> upd;   // (index, new count) of each touched (b, h), in order
    std::unordered_map<int, size_t> upd_at;
    ok.reserve(n);
    dst.reserve(n);
    for (size_t r = 0; r < n; ++r) {
        const int idx = recs[r].b * bl.H + recs[r].h;
        const int32_t cur = bl.shadow[idx];
        if (cur >= bl.Np) {
            headroom_full.fetch_add(1);
            continue;
        }
        bl.shadow[idx] = cur + 1;
        ok.push_back(recs + r);
        dst.push_back((int64_t)idx * bl.Np + cur);
        auto it = upd_at.find(idx);
        if (it == upd_at.end()) {
            upd_at[idx] = upd.size();
            upd.push_back(idx);
            upd.push_back(cur + 1);
        } else {
            upd[it->second + 1] = cur + 1;
        }
    }
    const int m = (int)(upd.size() / 2), cnt = (int)ok.size();
    if (cnt == 0) return;
    const size_t row = (size_t)D * sizeof(uint16_t);
    const size_t bytes = 2 * row * cnt + sizeof(int64_t) * cnt + upd.size() * sizeof(int32_t);
    // pinned buffer: wait until the copy out of its previous batch is done
    const int bi = next_buf;
    next_buf = (next_buf + 1) % kStagingBufs;
    if (cudaEventSynchronize(staging_ev[bi]) != cudaSuccess) {
        worker_error = "promotion worker: staging event failed";
        return;
    }
    if (bytes > staging_bytes[bi]) {
        if (staging[bi]) cudaFreeHost(staging[bi]);
        staging_bytes[bi] = std::max(bytes, 2 * staging_bytes[bi]);
        if (cudaHostAlloc((void**)&staging[bi], staging_bytes[bi], cudaHostAllocDefault) != cudaSuccess) {
            staging[bi] = nullptr;
            staging_bytes[bi] = 0;
            worker_error = "promotion worker: pinned staging allocation failed";
            return;
        }
    }
    if (bytes > dev_stage_bytes) {
        // the previous device buffer may still be read by queued scatters
        cudaStreamSynchronize(stream);
        if (dev_stage) cudaFree(dev_stage);
        dev_stage_bytes = std::max(bytes, 2 * dev_stage_bytes);
        if (cudaMalloc(&dev_stage, dev_stage_bytes) != cudaSuccess) {
            dev_stage = nullptr;
            dev_stage_bytes = 0;
            worker_error = "promotion worker: device staging allocation failed";
            return;
        }
    }
    uint8_t* st = staging[bi];
    uint16_t* sk = reinterpret_cast<uint16_t*>(st);
    uint16_t* sv = reinterpret_cast<uint16_t*>(st + row * cnt);
    for (int r = 0; r < cnt; ++r) {
        const size_t src = ((size_t)(ok[r]->b * a.H + ok[r]->h) * a.S + ok[r]->arc_local) * D;
        std::memcpy(sk + (size_t)r * D, a.k + src, row);
        std::memcpy(sv + (size_t)r * D, a.v + src, row);
    }
    std::memcpy(st + 2 * row * cnt, dst.data(), sizeof(int64_t) * cnt);
    std::memcpy(st + 2 * row * cnt + sizeof(int64_t) * cnt, upd.data(), upd.size() * sizeof(int32_t));
    if (cudaMemcpyAsync(dev_stage, st, bytes, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaEventRecord(staging_ev[bi], stream) != cudaSuccess ||
        fkv::promo_scatter(dev_stage, cnt, m, D, bl.near_k, bl.near_v, bl.near_valid, stream) != FKV_OK) {
        worker_error = "promotion worker: batch copy / scatter launch failed";
        return;
    }
    completed.fetch_add((uint64_t)cnt);
}

FkvPromo::~FkvPromo() {
    running = false;
    cv.notify_all();
    if (worker.joinable()) worker.join();
    if (cuda_ready) {
        cudaSetDevice(device);
        cudaStreamSynchronize(stream);
        for (auto& e : staging_ev) cudaEventDestroy(e);
        cudaEventDestroy(done);
        cudaStreamDestroy(stream);
        for (auto* b : staging)
            if (b) cudaFreeHost(b);
        if (dev_stage) cudaFree(dev_stage);
    }
    for (auto& a : archives) {
        if (a.map_k) munmap(a.map_k, a.map_bytes);
        if (a.map_v) munmap(a.map_v, a.map_bytes);
    }
}

namespace {

int check_layer(FkvPromo* p, int layer) {
    FKV_REQUIRE(p != nullptr, FKV_ERR_INVALID, "promotion pipeline is NULL");
    FKV_REQUIRE(layer >= 0 && layer < p->n_layers, FKV_ERR_INVALID,
                "layer %d out of range [0, %d)", layer, p->n_layers);
    return FKV_OK;
}

int set_archive_index(Archive& a, const int32_t* idx, int64_t len) {
    FKV_REQUIRE(idx != nullptr && len >= (int64_t)a.B * a.H * a.S, FKV_ERR_INVALID,
                "archive_idx has %lld entries, need B*H_kv*S_arc = %lld", (long long)len,
                (long long)a.B * a.H * a.S);
    a.pos_to_local.assign((size_t)a.B * a.H, {});
    for (int bh = 0; bh < a.B * a.H; ++bh) {
        auto& m = a.pos_to_local[bh];
        m.reserve(a.S);
        for (int i = 0; i < a.S; ++i) m[idx[(int64_t)bh * a.S + i]] = i;
    }
    return FKV_OK;
}

void* map_file(const char* path, size_t bytes, int& err) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) {
        err = 1;
        return nullptr;
    }
    struct stat sb;
    if (fstat(fd, &sb) != 0 || (size_t)sb.st_size < bytes) {
        close(fd);
        err = 2;
        return nullptr;
    }
    void* m = mmap(nullptr, bytes, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) {
        err = 3;
        return nullptr;
    }
    return m;
}

}  // namespace

extern "C" {

FkvPromo* fkv_promo_create(int32_t n_layers, int32_t cooldown_steps, int32_t max_per_drain,
                           int32_t device) {
    fkv::clear_error();
    if (n_layers <= 0 || cooldown_steps < 0 || max_per_drain < 0) {
        fkv::set_error("fkv_promo_create: n_layers=%d cooldown=%d budget=%d invalid", n_layers,
                       cooldown_steps, max_per_drain);
        return nullptr;
    }
    auto* p = new FkvPromo();
    p->n_layers = n_layers;
    p->cooldown = cooldown_steps;
    p->budget = max_per_drain;
    p->device = device;
    p->archives.resize(n_layers);
    p->blobs.resize(n_layers);
    p->worker = std::thread(&FkvPromo::run, p);
    return p;
}

int fkv_promo_register_archive(FkvPromo* p, int32_t layer, const char* path_k,
                               const char* path_v, int32_t B, int32_t H_kv, int32_t S_arc,
                               int32_t D, const int32_t* archive_idx, int64_t archive_idx_len) {
    fkv::clear_error();
    int rc = check_layer(p, layer);
    if (rc) return rc;
    FKV_REQUIRE(path_k && path_v && B > 0 && H_kv > 0 && S_arc >= 0 && D > 0, FKV_ERR_INVALID,
                "fkv_promo_register_archive: bad arguments");
    std::lock_guard<std::mutex> lk(p->mu);
    Archive& a = p->archives[layer];
    a = Archive{};
    a.B = B; a.H = H_kv; a.S = S_arc; a.D = D;
    rc = set_archive_index(a, archive_idx, archive_idx_len);
    if (rc) return rc;
    if (S_arc == 0) return FKV_OK;
    a.map_bytes = (size_t)B * H_kv * S_arc * D * sizeof(uint16_t);
    int err = 0;
    a.map_k = map_file(path_k, a.map_bytes, err);
    FKV_REQUIRE(a.map_k != nullptr, FKV_ERR_IO, "cannot map archive %s (error %d)", path_k, err);
    a.map_v = map_file(path_v, a.map_bytes, err);
    if (a.map_v == nullptr) {
        munmap(a.map_k, a.map_bytes);
        a.map_k = nullptr;
        fkv::set_error("cannot map archive %s (error %d)", path_v, err);
        return FKV_ERR_IO;
    }
    a.k = static_cast<const uint16_t*>(a.map_k);
    a.v = static_cast<const uint16_t*>(a.map_v);
    return FKV_OK;
}

int fkv_promo_register_archive_host(FkvPromo* p, int32_t layer, const uint16_t* host_k,
                                    const uint16_t* host_v, int32_t B, int32_t H_kv,
                                    int32_t S_arc, int32_t D, const int32_t* archive_idx,
                                    int64_t archive_idx_len) {
    fkv::clear_error();
    int rc = check_layer(p, layer);
    if (rc) return rc;
    FKV_REQUIRE((S_arc == 0 || (host_k && host_v)) && B > 0 && H_kv > 0 && S_arc >= 0 && D > 0,
                FKV_ERR_INVALID, "fkv_promo_register_archive_host: bad arguments");
    std::lock_guard<std::mutex> lk(p->mu);
    Archive& a = p->archives[layer];
    a = Archive{};
    a.B = B; a.H = H_kv; a.S = S_arc; a.D = D;
    rc = set_archive_index(a, archive_idx, archive_idx_len);
    if (rc) return rc;
    a.k = host_k;
    a.v = host_v;
    return FKV_OK;
}

int fkv_promo_register_blob(FkvPromo* p, int32_t layer, uint16_t* near_k, uint16_t* near_v,
                            int32_t* near_valid, int32_t B, int32_t H_kv, int32_t n_near_alloc,
                            int32_t D) {
    fkv::clear_error();
    int rc = check_layer(p, layer);
    if (rc) return rc;
    FKV_REQUIRE(near_k && near_v && near_valid && B > 0 && H_kv > 0 && n_near_alloc > 0 && D > 0,
                FKV_ERR_INVALID, "fkv_promo_register_blob: bad arguments");
    std::vector<int32_t> shadow((size_t)B * H_kv);
    FKV_CUDA_CHECK(cudaMemcpy(shadow.data(), near_valid, shadow.size() * sizeof(int32_t),
                              cudaMemcpyDeviceToHost));
    std::lock_guard<std::mutex> lk(p->mu);
    Blob& bl = p->blobs[layer];
    bl.near_k = near_k; bl.near_v = near_v; bl.near_valid = near_valid;
    bl.B = B; bl.H = H_kv; bl.Np = n_near_alloc; bl.D = D;
    bl.shadow = std::move(shadow);
    return FKV_OK;
}

// Filter order of PromotionPipeline::drain_spikes (promotion_pipeline.cpp:99-175):
// flag, GQA dedup, cooldown, far-local -> position, position dedup, archive
// lookup; at most max_per_drain records per call.
int fkv_promo_drain(FkvPromo* p, int32_t layer, const int32_t* flags, const int32_t* tokens,
                    const int32_t* far_idx, int32_t B, int32_t Hq, int32_t H_kv, int32_t n_far,
                    int32_t step) {
    fkv::clear_error();
    int rc = check_layer(p, layer);
    if (rc) return rc;
    FKV_REQUIRE(flags && tokens && B > 0 && Hq > 0 && H_kv > 0 && Hq % H_kv == 0 && n_far >= 0,
                FKV_ERR_INVALID, "fkv_promo_drain: bad arguments");
    FKV_REQUIRE(n_far == 0 || far_idx, FKV_ERR_INVALID, "fkv_promo_drain: far_idx is NULL");
    const Archive& a = p->archives[layer];
    if (!a.k || a.S == 0) return 0;   // no archive: nothing can be promoted
    const int G = Hq / H_kv;
    std::vector<char> seen((size_t)B * H_kv, 0);
    std::vector<Record> out;
    for (int b = 0; b < B && (int)out.size() < p->budget; ++b) {
        for (int hq = 0; hq < Hq && (int)out.size() < p->budget; ++hq) {
            const int flat = b * Hq + hq;
            if (flags[flat] == 0) continue;
            const int h = hq / G;
            if (seen[(size_t)b * H_kv + h]) continue;
            seen[(size_t)b * H_kv + h] = 1;
            p->detected.fetch_add(1);
            const uint64_t cd = ((uint64_t)layer << 40) | ((uint64_t)b << 20) | (uint64_t)h;
            auto it = p->last_step.find(cd);
            if (it != p->last_step.end() && step - it->second < p->cooldown) {
                p->cooled.fetch_add(1);
                continue;
            }
            p->last_step[cd] = step;
            const int fl = tokens[flat];
            if (fl < 0 || fl >= n_far) continue;
            const int32_t pos = far_idx[((int64_t)b * H_kv + h) * n_far + fl];
            if (!p->promoted.insert(std::make_tuple(layer, b, h, pos)).second) {
                p->deduplicated.fetch_add(1);
                continue;
            }
            if (b >= a.B || h >= a.H) continue;
            const auto& m = a.pos_to_local[(size_t)b * a.H + h];
            auto f = m.find(pos);
            if (f == m.end()) continue;
            out.push_back({layer, b, h, f->second});
            p->queued.fetch_add(1);
        }
    }
    if (!out.empty()) {
        {
            std::lock_guard<std::mutex> lk(p->mu);
            for (auto& r : out) p->queue.push_back(r);
        }
        p->cv.notify_one();
    }
    return (int)out.size();
}

int fkv_promo_flush(FkvPromo* p, void* stream, int32_t timeout_ms) {
    fkv::clear_error();
    FKV_REQUIRE(p != nullptr, FKV_ERR_INVALID, "promotion pipeline is NULL");
    {
        std::unique_lock<std::mutex> lk(p->mu);
        const bool ok = p->idle_cv.wait_for(lk, std::chrono::milliseconds(timeout_ms),
                                            [&] { return p->queue.empty() && !p->busy; });
        FKV_REQUIRE(ok, FKV_ERR_TIMEOUT, "fkv_promo_flush: queue not drained in %d ms",
                    timeout_ms);
        FKV_REQUIRE(p->worker_error.empty(), FKV_ERR_CUDA, "%s", p->worker_error.c_str());
        if (!p->cuda_ready) return FKV_OK;   // nothing was ever copied
        FKV_CUDA_CHECK(cudaEventRecord(p->done, p->stream));
    }
    if (stream != nullptr) FKV_CUDA_CHECK(cudaStreamWaitEvent((cudaStream_t)stream, p->done, 0));
    else FKV_CUDA_CHECK(cudaEventSynchronize(p->done));
    return FKV_OK;
}

int fkv_promo_stats(FkvPromo* p, uint64_t* s) {
    fkv::clear_error();
    FKV_REQUIRE(p && s, FKV_ERR_INVALID, "fkv_promo_stats: NULL argument");
    s[0] = p->detected; s[1] = p->queued; s[2] = p->deduplicated;
    s[3] = p->cooled; s[4] = p->completed; s[5] = p->headroom_full;
    return FKV_OK;
}

int fkv_promo_stop(FkvPromo* p) {
    fkv::clear_error();
    FKV_REQUIRE(p != nullptr, FKV_ERR_INVALID, "promotion pipeline is NULL");
    p->running = false;
    p->cv.notify_all();
    if (p->worker.joinable()) p->worker.join();
    return FKV_OK;
}

void fkv_promo_destroy(FkvPromo* p) { delete p; }

}  // extern "C"
