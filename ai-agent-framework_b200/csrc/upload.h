// GGUF tensor upload (upload.cpp): the file mapped read-only, byte ranges
// copied into a ring of pinned stages by a small pool of host threads (one
// slice each, so the page-cache reads run in parallel), each stage sent to
// the device with one cudaMemcpyAsync while the threads fill the next.
// transformer.go:1122-1335 (loadWeights) reads every tensor with
// ReadTensorData and dequantises on the host; here the blocks travel as they
// are and the device retiles them.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <condition_variable>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace b2 {

class Uploader {
public:
    static constexpr int kStages = 4;
    static constexpr size_t kStageBytes = 32u << 20;

    // threads <= 0: a count from the host's cores (at most 8).
    Uploader(const char* path, cudaStream_t stream, int threads = 0);
    ~Uploader();
    Uploader(const Uploader&) = delete;
    Uploader& operator=(const Uploader&) = delete;

    bool ok() const { return err_.empty(); }
    const std::string& error() const { return err_; }
    bool mapped() const { return map_ != nullptr; }
    uint64_t file_bytes() const { return file_bytes_; }

    // Queue the copy of file bytes [off, off + n) to device memory dst on the
    // stream (returns once the bytes are in pinned stages; the device copies
    // may still run).  False (and error()) on a short file or a CUDA error.
    bool to_device(uint64_t off, size_t n, void* dst) { return to_device_window(off, n, n, 1, dst); }
    // The same for a window of `width` bytes of each of `rows` rows that
    // start `pitch` bytes apart from off (a column share of a matrix): the
    // windows land back to back at dst, only their bytes are read and sent.
    bool to_device_window(uint64_t off, uint64_t pitch, uint64_t width, uint64_t rows, void* dst);
    // Synchronous read of a small range into host memory.
    bool to_host(uint64_t off, size_t n, void* dst);
    // Wait for every queued device copy.
    bool finish();

    // time the host threads spent filling stages, and the bytes sent
    int64_t host_ns() const { return host_ns_; }
    uint64_t bytes() const { return bytes_; }
    int threads() const { return (int)parts_; }

private:
    // packed bytes [p, p + n) of the current window into dst, in parallel
    // over the pool
    void fill(uint8_t* dst, uint64_t p, size_t n);
    void worker(int id);
    bool read_range(uint8_t* dst, uint64_t off, size_t n);
    // packed bytes [p + b, p + e) of the current window into dst + b (one
    // thread's slice)
    bool read_packed(uint8_t* dst, uint64_t p, size_t b, size_t e);

    int fd_ = -1;
    const uint8_t* map_ = nullptr;
    uint64_t file_bytes_ = 0;
    cudaStream_t stream_;
    uint8_t* stage_[kStages] = {};
    cudaEvent_t ev_[kStages] = {};
    bool used_[kStages] = {};
    int next_ = 0;
    std::string err_;
    int64_t host_ns_ = 0;
    uint64_t bytes_ = 0;

    // the window being copied: packed byte q is file byte
    // win_off_ + (q / win_width_) * win_pitch_ + q % win_width_
    uint64_t win_off_ = 0, win_pitch_ = 1, win_width_ = 1;
    // pool: job = (dst, p, n) split into equal slices, slice i to thread i
    std::vector<std::thread> pool_;
    size_t parts_ = 1;  // threads sharing a stage: the pool plus the caller
    std::mutex mu_;
    std::condition_variable cv_job_, cv_done_;
    uint64_t job_gen_ = 0;
    int job_pending_ = 0;
    bool stop_ = false;
    bool job_fail_ = false;
    uint8_t* job_dst_ = nullptr;
    uint64_t job_p_ = 0;
    size_t job_n_ = 0;
};

}  // namespace b2
