// GGUF tensor upload: mapped file -> pinned stages (parallel host copies) ->
// device (one cudaMemcpyAsync per stage).  See upload.h.
#include "upload.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstring>

namespace b2 {

namespace {
constexpr size_t kInlineBytes = 1u << 20;  // below this a stage is filled by the calling thread alone
constexpr size_t kSliceAlign = 4096;

int64_t now_ns() {
    return std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
        .count();
}
}  // namespace

Uploader::Uploader(const char* path, cudaStream_t stream, int threads) : stream_(stream) {
    fd_ = open(path, O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) {
        err_ = std::string("open model file: ") + path;
        return;
    }
    struct stat st {};
    if (fstat(fd_, &st) != 0) {
        err_ = std::string("stat model file: ") + path;
        return;
    }
    file_bytes_ = (uint64_t)st.st_size;
    if (file_bytes_ > 0) {
        void* p = mmap(nullptr, file_bytes_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (p != MAP_FAILED) {
            map_ = static_cast<const uint8_t*>(p);
            madvise(p, file_bytes_, MADV_SEQUENTIAL);
        }  // else: pread
    }
    for (int i = 0; i < kStages; i++) {
        if (cudaMallocHost(&stage_[i], kStageBytes) != cudaSuccess) {
            stage_[i] = nullptr;
            err_ = "pinned staging allocation failed";
            return;
        }
        if (cudaEventCreateWithFlags(&ev_[i], cudaEventDisableTiming) != cudaSuccess) {
            ev_[i] = nullptr;
            err_ = "event creation failed";
            return;
        }
    }
    if (threads <= 0) {
        const unsigned hc = std::max(1u, std::thread::hardware_concurrency());
        threads = (int)std::min(8u, std::max(1u, hc / 2));
    }
    parts_ = (size_t)threads;  // read by the workers: fixed before they start
    for (int i = 1; i < threads; i++) pool_.emplace_back(&Uploader::worker, this, i);
}

Uploader::~Uploader() {
    {
        std::lock_guard<std::mutex> lk(mu_);
        stop_ = true;
    }
    cv_job_.notify_all();
    for (std::thread& t : pool_) t.join();
    for (int i = 0; i < kStages; i++) {
        if (ev_[i]) {
            if (used_[i]) cudaEventSynchronize(ev_[i]);
            cudaEventDestroy(ev_[i]);
        }
        if (stage_[i]) cudaFreeHost(stage_[i]);
    }
    if (map_) munmap(const_cast<uint8_t*>(map_), file_bytes_);
    if (fd_ >= 0) close(fd_);
}

bool Uploader::read_range(uint8_t* dst, uint64_t off, size_t n) {
    if (map_) {
        memcpy(dst, map_ + off, n);
        return true;
    }
    while (n > 0) {
        const ssize_t r = pread(fd_, dst, n, (off_t)off);
        if (r <= 0) return false;
        dst += r;
        off += (uint64_t)r;
        n -= (size_t)r;
    }
    return true;
}

bool Uploader::read_packed(uint8_t* dst, uint64_t p, size_t b, size_t e) {
    while (b < e) {
        const uint64_t q = p + b, r = q / win_width_, c = q - r * win_width_;
        const size_t n = (size_t)std::min<uint64_t>(win_width_ - c, e - b);
        if (!read_range(dst + b, win_off_ + r * win_pitch_ + c, n)) return false;
        b += n;
    }
    return true;
}

void Uploader::worker(int id) {
    uint64_t seen = 0;
    for (;;) {
        uint8_t* dst;
        uint64_t p;
        size_t n;
        {
            std::unique_lock<std::mutex> lk(mu_);
            cv_job_.wait(lk, [&] { return stop_ || job_gen_ != seen; });
            if (stop_) return;
            seen = job_gen_;
            dst = job_dst_;
            p = job_p_;
            n = job_n_;
        }
        const size_t slice = ((n + parts_ - 1) / parts_ + kSliceAlign - 1) / kSliceAlign * kSliceAlign;
        const size_t b = std::min(n, (size_t)id * slice), e = std::min(n, b + slice);
        const bool ok = read_packed(dst, p, b, e);
        {
            std::lock_guard<std::mutex> lk(mu_);
            if (!ok) job_fail_ = true;
            if (--job_pending_ == 0) cv_done_.notify_one();
        }
    }
}

void Uploader::fill(uint8_t* dst, uint64_t p, size_t n) {
    const int64_t t0 = now_ns();
    if (pool_.empty() || n < kInlineBytes) {
        if (!read_packed(dst, p, 0, n)) job_fail_ = true;
    } else {
        {
            std::lock_guard<std::mutex> lk(mu_);
            job_dst_ = dst;
            job_p_ = p;
            job_n_ = n;
            job_pending_ = (int)pool_.size();
            job_gen_++;
        }
        cv_job_.notify_all();
        const size_t slice = ((n + parts_ - 1) / parts_ + kSliceAlign - 1) / kSliceAlign * kSliceAlign;
        if (!read_packed(dst, p, 0, std::min(n, slice))) {
            std::lock_guard<std::mutex> lk(mu_);
            job_fail_ = true;
        }
        std::unique_lock<std::mutex> lk(mu_);
        cv_done_.wait(lk, [&] { return job_pending_ == 0; });
    }
    host_ns_ += now_ns() - t0;
}

bool Uploader::to_device_window(uint64_t off, uint64_t pitch, uint64_t width, uint64_t rows, void* dst) {
    if (!ok()) return false;
    if (rows == 0 || width == 0) return true;
    if (width > pitch) {
        err_ = "upload window wider than its row pitch";
        return false;
    }
    const uint64_t span = (rows - 1) * pitch + width;  // (rows - 1) * pitch < file size checked below
    if (off > file_bytes_ || rows - 1 > (file_bytes_ - off) / pitch || span > file_bytes_ - off) {
        err_ = "tensor data beyond the end of the file";
        return false;
    }
    if (width == pitch) {  // whole rows: one contiguous range
        width = pitch = span;
        rows = 1;
    }
    win_off_ = off;
    win_pitch_ = pitch;
    win_width_ = width;
    uint64_t p = 0;
    size_t n = (size_t)(rows * width);
    uint8_t* d = static_cast<uint8_t*>(dst);
    while (n > 0) {
        const size_t nb = std::min(n, kStageBytes);
        const int s = next_;
        if (used_[s] && cudaEventSynchronize(ev_[s]) != cudaSuccess) {
            err_ = "upload copy failed";
            return false;
        }
        fill(stage_[s], p, nb);
        if (job_fail_) {
            err_ = "short read while uploading tensors";
            return false;
        }
        if (cudaMemcpyAsync(d, stage_[s], nb, cudaMemcpyHostToDevice, stream_) != cudaSuccess ||
            cudaEventRecord(ev_[s], stream_) != cudaSuccess) {
            err_ = "upload copy failed";
            return false;
        }
        used_[s] = true;
        next_ = (next_ + 1) % kStages;
        p += nb;
        d += nb;
        n -= nb;
        bytes_ += nb;
    }
    return true;
}

bool Uploader::to_host(uint64_t off, size_t n, void* dst) {
    if (!ok()) return false;
    if (off > file_bytes_ || n > file_bytes_ - off) {
        err_ = "tensor data beyond the end of the file";
        return false;
    }
    if (!read_range(static_cast<uint8_t*>(dst), off, n)) {
        err_ = "short read while uploading tensors";
        return false;
    }
    return true;
}

bool Uploader::finish() {
    for (int i = 0; i < kStages; i++)
        if (used_[i] && cudaEventSynchronize(ev_[i]) != cudaSuccess) {
            err_ = "upload copy failed";
            return false;
        }
    return ok();
}

}  // namespace b2
