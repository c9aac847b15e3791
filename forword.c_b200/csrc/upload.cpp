// upload.cpp — see upload.h.
#include "upload.h"

#include <algorithm>
#include <chrono>
#include <cstring>

namespace fwb {

static double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

Uploader::~Uploader() {
    {
        std::lock_guard<std::mutex> lk(mu_);
        stop_ = true;
    }
    cv_.notify_all();
    for (auto &t : pool_) t.join();
    if (st_) cudaStreamSynchronize(st_);
    for (auto *p : stage_) cudaFreeHost(p);
    for (auto e : ev_) cudaEventDestroy(e);
}

bool Uploader::open(cudaStream_t st, size_t chunk, int n_stage, int threads) {
    st_ = st;
    chunk_ = chunk;
    t0_ = now_s();
    for (int i = 0; i < n_stage; ++i) {
        uint8_t *p = nullptr;
        cudaEvent_t e = nullptr;
        if (cudaMallocHost(&p, chunk) != cudaSuccess ||
            cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
            if (p) cudaFreeHost(p);
            err_ = "upload: pinned staging allocation failed";
            return false;
        }
        stage_.push_back(p);
        ev_.push_back(e);
        if (cudaEventRecord(e, st) != cudaSuccess) { err_ = "upload: event record failed"; return false; }
    }
    if (threads <= 0) {
        const unsigned hc = std::thread::hardware_concurrency();
        threads = (int)std::max(1u, std::min(8u, hc ? hc : 1u));
    }
    for (int i = 1; i < threads; ++i) pool_.emplace_back(&Uploader::worker, this, i);
    return true;
}

void Uploader::worker(int id) {
    uint64_t seen = 0;
    for (;;) {
        const Fill *f;
        uint64_t off, n;
        uint8_t *dst;
        {
            std::unique_lock<std::mutex> lk(mu_);
            cv_.wait(lk, [&] { return stop_ || job_gen_ != seen; });
            if (stop_) return;
            seen = job_gen_;
            f = job_fill_;
            off = job_off_;
            n = job_n_;
            dst = job_dst_;
        }
        const uint64_t parts = pool_.size() + 1;
        const uint64_t a = n * (uint64_t)id / parts, b = n * (uint64_t)(id + 1) / parts;
        if (b > a) (*f)(off + a, b - a, dst + a);
        {
            std::lock_guard<std::mutex> lk(mu_);
            if (--job_left_ == 0) done_cv_.notify_one();
        }
    }
}

void Uploader::parallel_fill(const Fill &fill, uint64_t off, uint64_t n, uint8_t *dst) {
    if (pool_.empty() || n < (uint64_t(1) << 20)) {  // small pieces: this thread alone
        fill(off, n, dst);
        return;
    }
    const uint64_t parts = pool_.size() + 1;
    {
        std::lock_guard<std::mutex> lk(mu_);
        job_fill_ = &fill;
        job_off_ = off;
        job_n_ = n;
        job_dst_ = dst;
        job_left_ = (int)pool_.size();
        ++job_gen_;
    }
    cv_.notify_all();
    const uint64_t b = n / parts;  // part 0 here
    if (b) fill(off, b, dst);
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return job_left_ == 0; });
}

bool Uploader::add(uint8_t *dev_dst, uint64_t len, const Fill &fill) {
    uint64_t done = 0;
    while (done < len) {
        if (fill_ == 0 && cudaEventSynchronize(ev_[cur_]) != cudaSuccess) {  // the stage is free again
            err_ = "upload: staging event failed";
            return false;
        }
        const uint64_t take = std::min<uint64_t>(len - done, chunk_ - fill_);
        parallel_fill(fill, done, take, stage_[cur_] + fill_);
        pieces_.push_back({dev_dst + done, fill_, (size_t)take});
        fill_ += take;
        done += take;
        bytes_ += take;
        if (fill_ == chunk_ && !flush()) return false;
    }
    return true;
}

bool Uploader::flush() {
    if (fill_ == 0) return true;
    for (const Piece &p : pieces_)
        if (cudaMemcpyAsync(p.dst, stage_[cur_] + p.so, p.len, cudaMemcpyHostToDevice, st_) != cudaSuccess) {
            err_ = "upload: host-to-device copy failed";
            return false;
        }
    if (cudaEventRecord(ev_[cur_], st_) != cudaSuccess) { err_ = "upload: event record failed"; return false; }
    pieces_.clear();
    fill_ = 0;
    cur_ = (cur_ + 1) % (int)stage_.size();
    return true;
}

bool Uploader::finish() {
    if (!flush()) return false;
    if (cudaStreamSynchronize(st_) != cudaSuccess) { err_ = "upload: copies failed"; return false; }
    seconds_ = now_s() - t0_;
    return true;
}

}  // namespace fwb
