// lc_load.cu -- the model loaders' upload path: GGUF tensors from the reader's
// file mapping into one device allocation per model, through pinned staging.
//
// The reference reads each tensor with read_exact into a Vec (src/gguf.rs:415-421)
// and copies it into a host-visible buffer (src/model.rs:174-184), one tensor at
// a time.  Here every tensor a model uses is laid out in one device image
// (256-byte aligned, file order) and streamed in 64 MiB chunks: the host fills
// a pinned buffer from the mapping (several threads, so a cold file's page
// faults are taken in parallel) while the copy engine drains the previous one.
// F16 / BF16 tensors are decoded to f32 behind the copies on the same stream.
#include <algorithm>
#include <thread>
#include <vector>

#include "lc_internal.cuh"

namespace {

#define LC_TRY(expr)                \
    do {                            \
        int _s = (expr);            \
        if (_s != LC_OK) return _s; \
    } while (0)

// Host copy of n bytes split over up to `threads` threads.
void par_copy(uint8_t *dst, const uint8_t *src, size_t n, unsigned threads) {
    constexpr size_t kMinSlice = 4u << 20;
    const unsigned t = (unsigned)std::min<size_t>(threads, std::max<size_t>(1, n / kMinSlice));
    if (t <= 1) {
        memcpy(dst, src, n);
        return;
    }
    const size_t slice = (n / t + 4095) & ~(size_t)4095;
    std::vector<std::thread> pool;
    for (unsigned i = 1; i < t; i++) {
        const size_t a = std::min(n, i * slice), b = std::min(n, (i + 1) * slice);
        if (a < b) pool.emplace_back([=] { memcpy(dst + a, src + a, b - a); });
    }
    memcpy(dst, src, std::min(n, slice));
    for (auto &th : pool) th.join();
}

// One tensor of the device image: bytes [src, src + bytes) of the mapping go
// to image offset `at`; F16 / BF16 tensors are then decoded to f32 at `f32_at`.
struct Piece {
    lc::DevTensor *slot;
    int dtype;
    const uint8_t *src;
    uint64_t bytes, n_el, at, f32_at;
    uint64_t shape[4];
    uint32_t n_dims;
};

// Pinned staging of the device image: kBufs buffers of kChunk bytes; a buffer
// is refilled only after the copy that read it has completed (its event).
class Stager {
  public:
    static constexpr size_t kChunk = 64ull << 20;
    static constexpr int kBufs = 3;

    ~Stager() {
        for (int i = 0; i < kBufs; i++) {
            if (done_[i]) {
                cudaEventSynchronize(done_[i]);
                cudaEventDestroy(done_[i]);
            }
            if (buf_[i]) cudaFreeHost(buf_[i]);
        }
    }
    int init(cudaStream_t st, size_t image_bytes) {
        st_ = st;
        const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
        threads_ = std::min(8u, std::max(1u, hw / 2));
        const int n = (int)std::min<size_t>(kBufs, (image_bytes + kChunk - 1) / kChunk);
        for (int i = 0; i < n; i++) {
            LC_CUDA(cudaHostAlloc((void **)&buf_[i], kChunk, cudaHostAllocDefault));
            LC_CUDA(cudaEventCreateWithFlags(&done_[i], cudaEventDisableTiming));
        }
        nbuf_ = std::max(n, 1);
        return LC_OK;
    }
    // Copy the image [0, image_bytes) described by `pieces` (sorted by `at`,
    // non-overlapping) to dev; alignment gaps are left as they are.
    int upload(uint8_t *dev, const std::vector<Piece> &pieces, size_t image_bytes) {
        size_t first = 0;
        for (size_t c0 = 0, chunk = 0; c0 < image_bytes; c0 += kChunk, chunk++) {
            const size_t c1 = std::min(image_bytes, c0 + kChunk);
            const int b = (int)(chunk % (size_t)nbuf_);
            LC_CUDA(cudaEventSynchronize(done_[b]));
            while (first < pieces.size() && pieces[first].at + pieces[first].bytes <= c0) first++;
            for (size_t i = first; i < pieces.size() && pieces[i].at < c1; i++) {
                const Piece &p = pieces[i];
                const size_t a = std::max<size_t>(c0, p.at), e = std::min<size_t>(c1, p.at + p.bytes);
                if (a < e) par_copy(buf_[b] + (a - c0), p.src + (a - p.at), e - a, threads_);
            }
            LC_CUDA(cudaMemcpyAsync(dev + c0, buf_[b], c1 - c0, cudaMemcpyHostToDevice, st_));
            LC_CUDA(cudaEventRecord(done_[b], st_));
        }
        return LC_OK;
    }

  private:
    cudaStream_t st_ = nullptr;
    uint8_t *buf_[kBufs] = {};
    cudaEvent_t done_[kBufs] = {};
    int nbuf_ = 1;
    unsigned threads_ = 1;
};

}  // namespace

int lc::load_tensors(lc_ctx *ctx, lc_gguf *g, const std::function<DevTensor *(const char *)> &slot, uint32_t flags,
                     std::vector<void *> *allocs) {
    LC_TRY(lc_use_device(ctx));
    std::vector<Piece> pieces;
    uint64_t image = 0;
    auto align = [](uint64_t v) { return (v + 255) & ~(uint64_t)255; };
    for (uint64_t i = 0; i < lc_gguf_tensor_count(g); i++) {
        const char *name;
        int dtype;
        uint32_t n_dims;
        uint64_t shape[4], nbytes;
        LC_TRY(lc_gguf_tensor_info(g, i, &name, &dtype, &n_dims, shape, nullptr, &nbytes));
        DevTensor *w = slot(name);
        if (!w) continue;  // tensors the model does not use are skipped, like the reference's loaders
        const uint64_t be = lc_type_block_elements(dtype), bb = lc_type_block_bytes(dtype);
        LC_REQUIRE(be && bb, LC_ERR_UNSUPPORTED, "lc_load: %s has unsupported type %d", name, dtype);
        const void *src;
        LC_TRY(lc_gguf_tensor_data(g, i, &src, nullptr));
        image = align(image);
        Piece p{w, dtype, (const uint8_t *)src, nbytes, nbytes / bb * be, image, 0, {}, n_dims};
        for (int d = 0; d < 4; d++) p.shape[d] = shape[d];
        pieces.push_back(p);
        image += nbytes;
    }
    uint64_t total = align(image);
    for (Piece &p : pieces)
        if (p.dtype == LC_F16 || p.dtype == LC_BF16) {
            p.f32_at = total;
            total = align(total + p.n_el * 4);
        }
    if (pieces.empty()) return LC_OK;
    void *arena = nullptr;
    cudaError_t e = cudaMalloc(&arena, total);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return lc_fail(LC_ERR_OOM, "lc_load: cudaMalloc(%llu): %s", (unsigned long long)total, cudaGetErrorString(e));
    }
    allocs->push_back(arena);
    uint8_t *dev = (uint8_t *)arena;
    {
        Stager stager;
        LC_TRY(stager.init(ctx->stream, image));
        LC_TRY(stager.upload(dev, pieces, image));
        for (const Piece &p : pieces) {
            DevTensor *w = p.slot;
            if (p.dtype == LC_F16 || p.dtype == LC_BF16) {
                // dequant_to_f32 rules (src/dflash.rs:351-378, :437-462), or bfloat16 on request
                const bool native = p.dtype == LC_BF16 && (flags & LC_LOAD_BF16_NATIVE);
                LC_TRY(dequant_f32(ctx, p.dtype, dev + p.at, p.bytes, p.n_el, (float *)(dev + p.f32_at), native));
                w->ptr = dev + p.f32_at;
                w->bytes = (size_t)p.n_el * 4;
                w->dtype = LC_F32;
            } else {
                w->ptr = dev + p.at;
                w->bytes = (size_t)p.bytes;
                w->dtype = p.dtype;
            }
            w->n_el = p.n_el;
            w->n_dims = p.n_dims;
            for (int d = 0; d < 4; d++) w->shape[d] = p.shape[d];
        }
        // the stager's destructor waits for its buffers before freeing them
    }
    LC_CUDA(cudaStreamSynchronize(ctx->stream));
    return LC_OK;
}
