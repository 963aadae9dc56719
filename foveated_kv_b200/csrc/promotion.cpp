// Spike drain + promotion of exact fp16 rows into near-tier headroom.
//
// Host side of the closed loop of the reference's PromotionPipeline
// (csrc/promotion_pipeline.cpp:20-248): drain_spikes filters the fused
// kernel's per-head spike flags (GQA dedup, cooldown, position dedup, budget)
// and queues records; one worker std::thread per pipeline copies the exact
// fp16 K/V rows of each record from a host archive (mmapped file or caller
// memory) through pinned staging into slot near_valid[b, h] of the device
// near tier with cudaMemcpyAsync on its own stream, then writes the new count
// with a second copy on the same stream.  Stream order makes the count visible
// only after the row it covers, so a decode launch that reads near_valid sees
// either the old count or the new count with its row in place.
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

constexpr int kStagingSlots = 64;

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

    // device resources, created by the worker on first use
    bool cuda_ready = false;
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    uint8_t* staging = nullptr;                 // pinned, kStagingSlots slots
    size_t slot_bytes = 0;
    cudaEvent_t slot_ev[kStagingSlots] = {};
    int next_slot = 0;
    std::string worker_error;

    ~FkvPromo();
    void run();
    bool ensure_cuda(size_t need_slot_bytes);
    void promote(const Record& r);
};

void FkvPromo::run() {
    while (true) {
        Record r;
        {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return !queue.empty() || !running.load(); });
            if (queue.empty()) break;   // stopping and drained
            r = queue.front();
            queue.pop_front();
            busy = true;
        }
        promote(r);
        {
            std::lock_guard<std::mutex> lk(mu);
            busy = false;
        }
        idle_cv.notify_all();
    }
    idle_cv.notify_all();
}

bool FkvPromo::ensure_cuda(size_t need) {
    if (cuda_ready && need <= slot_bytes) return true;
    if (cudaSetDevice(device) != cudaSuccess) return false;
    if (!cuda_ready) {
        if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess) return false;
        if (cudaEventCreateWithFlags(&done, cudaEventDisableTiming) != cudaSuccess) return false;
        for (auto& e : slot_ev)
            if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return false;
    }
    if (need > slot_bytes) {
        cudaStreamSynchronize(stream);
        if (staging) cudaFreeHost(staging);
        slot_bytes = (need + 255) & ~(size_t)255;
        if (cudaHostAlloc((void**)&staging, slot_bytes * kStagingSlots, cudaHostAllocDefault) !=
            cudaSuccess) {
            staging = nullptr;
            slot_bytes = 0;
            return false;
        }
    }
    cuda_ready = true;
    return true;
}

void FkvPromo::promote(const Record& r) {
    Archive& a = archives[r.layer];
    Blob& bl = blobs[r.layer];
    if (!a.k || !bl.near_k) return;   // nothing to promote into (reference: :215-216)
    const int idx = r.b * bl.H + r.h;
    const int32_t cur = bl.shadow[idx];
    if (cur >= bl.Np) {
        headroom_full.fetch_add(1);
        return;
    }
    const size_t row = (size_t)a.D * sizeof(uint16_t);
    if (!ensure_cuda(2 * row + 16)) {
        worker_error = "promotion worker: CUDA setup failed";
        return;
    }
    const int slot = next_slot;
    next_slot = (next_slot + 1) % kStagingSlots;
    cudaEventSynchronize(slot_ev[slot]);   // previous copies out of this slot are done
    uint8_t* st = staging + (size_t)slot * slot_bytes;
    const size_t src = ((size_t)(r.b * a.H + r.h) * a.S + r.arc_local) * a.D;
    std::memcpy(st, a.k + src, row);
    std::memcpy(st + row, a.v + src, row);
    int32_t* cnt = reinterpret_cast<int32_t*>(st + 2 * row);
    *cnt = cur + 1;
    const size_t dst = ((size_t)idx * bl.Np + cur) * bl.D;
    cudaMemcpyAsync(bl.near_k + dst, st, row, cudaMemcpyHostToDevice, stream);
    cudaMemcpyAsync(bl.near_v + dst, st + row, row, cudaMemcpyHostToDevice, stream);
    cudaMemcpyAsync(bl.near_valid + idx, cnt, sizeof(int32_t), cudaMemcpyHostToDevice, stream);
    cudaEventRecord(slot_ev[slot], stream);
    bl.shadow[idx] = cur + 1;
    completed.fetch_add(1);
}

FkvPromo::~FkvPromo() {
    running = false;
    cv.notify_all();
    if (worker.joinable()) worker.join();
    if (cuda_ready) {
        cudaSetDevice(device);
        cudaStreamSynchronize(stream);
        for (auto& e : slot_ev) cudaEventDestroy(e);
        cudaEventDestroy(done);
        cudaStreamDestroy(stream);
        if (staging) cudaFreeHost(staging);
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
