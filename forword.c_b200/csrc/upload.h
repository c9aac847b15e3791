// upload.h — host-to-HBM upload of a model's tensors at open time.
//
// The reference reads weights straight from its mmap on every token
// (tensor_data.c:25-62); here every tensor is copied once into the device
// arena.  Bytes are produced into a ring of page-locked staging buffers by
// several host threads in parallel (a plain copy out of the GGUF mapping,
// or, under tensor parallelism, the packing of a rank's slice) while earlier
// buffers are in flight to the device with cudaMemcpyAsync.
#pragma once
#include <cuda_runtime.h>

#include <condition_variable>
#include <cstdint>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace fwb {

class Uploader {
public:
    // fill(off, n, dst): write bytes [off, off + n) of the piece to dst.
    // Called concurrently on disjoint ranges.
    using Fill = std::function<void(uint64_t off, uint64_t n, uint8_t *dst)>;

    ~Uploader();
    bool open(cudaStream_t st, size_t chunk = size_t(64) << 20, int n_stage = 4, int threads = 0);
    // Queue `len` bytes for dev_dst.  Returns false on a CUDA error.
    bool add(uint8_t *dev_dst, uint64_t len, const Fill &fill);
    // Flush and wait for every copy.  Returns false on a CUDA error.
    bool finish();
    const std::string &error() const { return err_; }
    double seconds() const { return seconds_; }
    uint64_t bytes() const { return bytes_; }

private:
    struct Piece { uint8_t *dst; size_t so, len; };
    bool flush();
    void parallel_fill(const Fill &fill, uint64_t off, uint64_t n, uint8_t *dst);
    void worker(int id);

    cudaStream_t st_ = nullptr;
    size_t chunk_ = 0, fill_ = 0;
    int cur_ = 0;
    std::vector<uint8_t *> stage_;
    std::vector<cudaEvent_t> ev_;
    std::vector<Piece> pieces_;
    std::string err_;
    double seconds_ = 0, t0_ = 0;
    uint64_t bytes_ = 0;
    // worker pool: job = (fill, off, n, dst) split into nthreads contiguous parts
    std::vector<std::thread> pool_;
    std::mutex mu_;
    std::condition_variable cv_, done_cv_;
    const Fill *job_fill_ = nullptr;
    uint64_t job_off_ = 0, job_n_ = 0;
    uint8_t *job_dst_ = nullptr;
    uint64_t job_gen_ = 0;
    int job_left_ = 0;
    bool stop_ = false;
};

}  // namespace fwb
