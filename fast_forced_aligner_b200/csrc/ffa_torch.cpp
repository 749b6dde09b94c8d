// ffa_torch.cpp -- thin PyTorch operator layer over the C ABI (libffa_b200.so).
//
// Registers torch.ops.ffa_b200.{align, align_packed, emission_validity,
// check_targets, token_spans, row_logsumexp, align_stream}.  It mirrors the
// reference's op layer (alignment.cu:893-1061, TORCH_LIBRARY at
// alignment.cu:1064-1070): tensor metadata checks, stream lifetime
// protection (recordStream on borrowed inputs) and output allocation from
// the caching allocator.  Everything below the ffa_* calls is plain pointers
// and sizes.  Per call it makes two caching-allocator requests (one block
// holds every output tensor, one the workspace) and stages descriptors in a
// reused pinned host buffer, so the host cost stays a few microseconds.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <climits>
#include <initializer_list>
#include <optional>
#include <tuple>
#include <vector>

#include "ffa_b200.h"

namespace {

void check_status(int rc) {
  if (rc == FFA_OK) return;
  if (rc == FFA_ERR_INVALID_ARGUMENT || rc == FFA_ERR_UNSUPPORTED)
    TORCH_CHECK_VALUE(false, ffa_last_error());
  TORCH_CHECK(false, "fast_forced_aligner_b200: ", ffa_last_error());
}

// Protect a borrowed allocation against reuse by another stream while this
// call's kernels read it (alignment.cu:977-980).  Consecutive records that
// share one storage are recorded once.
struct StreamRecorder {
  c10::cuda::CUDAStream stream;
  const void* last = nullptr;
  void operator()(const at::Tensor& t) {
    if (t.numel() == 0) return;
    const void* key = t.storage().data_ptr().get();
    if (key == last) return;
    last = key;
    c10::cuda::CUDACachingAllocator::recordStream(t.storage().data_ptr(), stream);
  }
};

// Host staging for the descriptor upload: pinned, so that the upload is a
// plain DMA (from pageable memory the driver copies the bytes itself first,
// which costs tens of microseconds of host time).  Each thread keeps a small
// ring of pinned buffers per device; a buffer is reused once the event
// recorded after its upload has completed, and a buffer is (re)allocated only
// while the ring grows to the batch sizes in use.
class PinnedStaging {
 public:
  // A buffer of at least `bytes`, not in use by an upload still pending.
  void* acquire(size_t bytes) {
    for (int tries = 0; tries < 2 * kSlots; ++tries) {
      Slot& slot = slots_[next_];
      current_ = next_;
      next_ = (next_ + 1) % kSlots;
      if (slot.pending && cudaEventQuery(slot.done) != cudaSuccess) continue;
      slot.pending = false;
      if (slot.capacity < bytes) {
        // Pinning memory is slow (milliseconds) and can synchronise: grow
        // every idle buffer now, so that later calls of this size never do.
        for (Slot& other : slots_) {
          if (other.capacity >= bytes || (&other != &slot && other.pending &&
                                          cudaEventQuery(other.done) != cudaSuccess))
            continue;
          other.pending = false;
          grow(other, bytes);
        }
      }
      if (slot.done == nullptr)
        TORCH_CHECK(cudaEventCreateWithFlags(&slot.done, cudaEventDisableTiming) == cudaSuccess,
                    "fast_forced_aligner_b200: cannot create a staging event");
      return slot.ptr;
    }
    // Every buffer still pending: wait for the oldest.
    Slot& slot = slots_[next_];
    cudaEventSynchronize(slot.done);
    slot.pending = false;
    return acquire(bytes);
  }
  // Marks the buffer handed out last as in use until the stream passes here.
  void release(cudaStream_t stream) {
    Slot& slot = slots_[current_];
    if (cudaEventRecord(slot.done, stream) == cudaSuccess) slot.pending = true;
  }

 private:
  static constexpr int kSlots = 4;
  struct Slot {
    void* ptr = nullptr;
    size_t capacity = 0;
    cudaEvent_t done = nullptr;
    bool pending = false;
  };
  static void grow(Slot& slot, size_t bytes) {
    if (slot.ptr != nullptr) cudaFreeHost(slot.ptr);
    slot.ptr = nullptr;
    slot.capacity = 0;
    const size_t cap = std::max<size_t>(bytes, size_t{64} << 10);
    TORCH_CHECK(cudaHostAlloc(&slot.ptr, cap, cudaHostAllocPortable) == cudaSuccess,
                "fast_forced_aligner_b200: cannot allocate pinned staging");
    slot.capacity = cap;
  }
  Slot slots_[kSlots];
  int next_ = 0, current_ = 0;
};

PinnedStaging& staging_for(int device) {
  thread_local PinnedStaging rings[64];
  TORCH_CHECK(device >= 0 && device < 64, "fast_forced_aligner_b200: device index out of range");
  return rings[device];
}

// Device scratch from the caching allocator on the current stream; returned
// to the cache (stream-ordered) when the DataPtr goes away.
c10::DataPtr device_scratch(size_t bytes) {
  return c10::cuda::CUDACachingAllocator::get()->allocate(std::max<size_t>(bytes, 256));
}

// Several output tensors carved from one caching-allocator block: each is a
// contiguous tensor on a shared storage at a 256-byte aligned offset, built
// without a dispatcher round trip per tensor.
class OutputBlock {
 public:
  template <typename T>
  void add(std::initializer_list<int64_t> sizes) {
    int64_t n = 1;
    for (int64_t v : sizes) n *= v;
    specs_.push_back({bytes_, std::vector<int64_t>(sizes), caffe2::TypeMeta::Make<T>()});
    bytes_ = (bytes_ + static_cast<size_t>(n) * sizeof(T) + 255) / 256 * 256;
  }
  std::vector<at::Tensor> allocate() {
    auto* allocator = c10::cuda::CUDACachingAllocator::get();
    c10::Storage storage(c10::Storage::use_byte_size_t(), static_cast<int64_t>(bytes_),
                         allocator->allocate(std::max<size_t>(bytes_, 256)), allocator, false);
    std::vector<at::Tensor> out;
    out.reserve(specs_.size());
    for (const auto& spec : specs_) {
      auto t = at::detail::make_tensor<c10::TensorImpl>(
          c10::Storage(storage), c10::DispatchKeySet(c10::DispatchKey::CUDA), spec.dtype);
      t.unsafeGetTensorImpl()->set_sizes_contiguous(spec.sizes);
      t.unsafeGetTensorImpl()->set_storage_offset(static_cast<int64_t>(spec.offset / spec.dtype.itemsize()));
      out.push_back(std::move(t));
    }
    return out;
  }

 private:
  struct Spec {
    size_t offset;
    std::vector<int64_t> sizes;
    caffe2::TypeMeta dtype;
  };
  std::vector<Spec> specs_;
  size_t bytes_ = 0;
};

const uint8_t* check_mask(const std::optional<at::Tensor>& validity, const c10::Device& device,
                          int64_t count, StreamRecorder& rec) {
  if (!validity.has_value()) return nullptr;
  const auto& mask = *validity;
  TORCH_CHECK_VALUE(mask.device() == device && mask.scalar_type() == at::kBool && mask.dim() == 1 &&
                        mask.numel() == count && mask.is_contiguous(),
                    "emission_validity must be contiguous CUDA bool [batch] on the input device");
  rec(mask);
  return reinterpret_cast<const uint8_t*>(mask.data_ptr<bool>());
}

std::tuple<std::vector<at::Tensor>, std::vector<int64_t>> run_align(
    const std::vector<ffa_record>& recs, const c10::Device& device, int64_t mode,
    const uint8_t* mask, bool check_inputs, c10::cuda::CUDAStream stream,
    std::vector<int64_t> lengths) {
  const int64_t count = static_cast<int64_t>(recs.size());
  // mode 0 conventional, 1 optimized, 2 optimized on the chunked route only,
  // 3 optimized on the window route wherever it applies.
  const int cmode = mode == 0 ? FFA_MODE_CONVENTIONAL : FFA_MODE_OPTIMIZED;
  const int flags = (check_inputs ? FFA_FLAG_CHECK_INPUTS : 0) | (mode == 2 ? FFA_FLAG_PIECE_ROUTE : 0) |
                    (mode == 3 ? FFA_FLAG_WINDOW_ROUTE : 0);
  ffa_sizes sizes{};
  check_status(ffa_align_query(recs.data(), count, cmode, flags, &sizes));

  const int64_t N = sizes.total_frames;
  int64_t max_frames = 0;
  for (const auto& r : recs) max_frames = std::max(max_frames, r.frames);
  const bool reuse = cmode == FFA_MODE_OPTIMIZED && max_frames >= 2048;
  OutputBlock block;
  block.add<int64_t>({N});                        // labels
  block.add<float>({N});                          // scores
  block.add<int32_t>({count});                    // status
  block.add<float>({count});                      // objective
  block.add<int32_t>({count});                    // stitched
  block.add<int32_t>({count});                    // repair_passes
  block.add<int64_t>({count});                    // repaired_frames
  block.add<int64_t>({count, 3});                 // shortcut_stats
  block.add<int32_t>({count, 3});                 // routing_stats
  block.add<int64_t>({reuse ? count : 0, 4});     // reuse_stats
  std::vector<at::Tensor> t = block.allocate();
  auto workspace = device_scratch(sizes.workspace_bytes);
  ffa_outputs out{t[0].data_ptr<int64_t>(), t[1].data_ptr<float>(), t[2].data_ptr<int32_t>(),
                  t[3].data_ptr<float>(), t[4].data_ptr<int32_t>(), t[5].data_ptr<int32_t>(),
                  t[6].data_ptr<int64_t>(), t[7].data_ptr<int64_t>(), t[8].data_ptr<int32_t>(),
                  reuse ? t[9].data_ptr<int64_t>() : nullptr};
  PinnedStaging& staging = staging_for(device.index());
  const int rc = ffa_align(recs.data(), count, cmode, flags, mask, &out, staging.acquire(sizes.staging_bytes),
                           sizes.staging_bytes, workspace.get(), std::max<size_t>(sizes.workspace_bytes, 256),
                           reinterpret_cast<ffa_stream_t>(stream.stream()));
  if (rc == FFA_OK) staging.release(stream.stream());
  check_status(rc);
  return {std::move(t), std::move(lengths)};
}

void check_mode(int64_t mode) {
  TORCH_CHECK_VALUE(mode >= 0 && mode <= 3, "mode must be 'optimized' or 'conventional'");
}

// Input format (ffa_input_format) and the dtype it stores: fp32
// log-probabilities, fp32 logits, bf16 logits.
at::ScalarType format_dtype(int64_t fmt) {
  TORCH_CHECK_VALUE(fmt >= FFA_INPUT_LOG_PROBS && fmt <= FFA_INPUT_LOGITS_BF16, "unknown input format");
  return fmt == FFA_INPUT_LOGITS_BF16 ? at::kBFloat16 : at::kFloat;
}
const char* format_message(int64_t fmt, bool packed) {
  if (fmt == FFA_INPUT_LOGITS_BF16)
    return packed ? "inputs must be contiguous CUDA bfloat16 [N,V] and int64 [M] on one device"
                  : "inputs must be contiguous CUDA bfloat16 [T,V] and int64 [U] on one device";
  return packed ? "inputs must be contiguous CUDA float32 [N,V] and int64 [M] on one device"
                : "inputs must be contiguous CUDA float32 [T,V] and int64 [U] on one device";
}

// align(Tensor[] emissions, Tensor[] targets, int[] blanks, int mode,
//       Tensor? emission_validity, bool check_inputs, int fmt) -> (Tensor[], int[])
// fmt: ffa_input_format (1, 2: the emissions are logits, aligned as their
// log_softmax).
std::tuple<std::vector<at::Tensor>, std::vector<int64_t>> align(
    at::TensorList emissions, at::TensorList targets, at::IntArrayRef blanks, int64_t mode,
    const std::optional<at::Tensor>& emission_validity, bool check_inputs, int64_t fmt) {
  check_mode(mode);
  const at::ScalarType dtype = format_dtype(fmt);
  const char* msg = format_message(fmt, false);
  const int64_t count = static_cast<int64_t>(emissions.size());
  TORCH_CHECK_VALUE(count > 0 && count <= FFA_MAX_RECORDS &&
                        static_cast<int64_t>(targets.size()) == count &&
                        static_cast<int64_t>(blanks.size()) == count,
                    "provide 1..65535 matching emissions and targets");
  const auto device = emissions[0].device();
  TORCH_CHECK_VALUE(device.is_cuda(), msg);
  c10::cuda::CUDAGuard guard(device);
  const auto stream = c10::cuda::getCurrentCUDAStream();
  StreamRecorder rec{stream};
  std::vector<ffa_record> recs(count);
  std::vector<int64_t> lengths(count);
  for (int64_t i = 0; i < count; ++i) {
    const auto& e = emissions[i];
    const auto& t = targets[i];
    TORCH_CHECK_VALUE(e.device() == device && t.device() == device &&
                          e.scalar_type() == dtype && t.scalar_type() == at::kLong &&
                          e.dim() == 2 && t.dim() == 1 && e.is_contiguous() && t.is_contiguous(),
                      msg);
    TORCH_CHECK_VALUE(e.size(0) > 0 && e.size(0) <= INT_MAX && e.size(1) > 0 &&
                          e.size(1) <= FFA_MAX_VOCAB && t.numel() <= FFA_MAX_TOKENS && blanks[i] >= 0 &&
                          blanks[i] < e.size(1),
                      "unsupported frame count, vocabulary, target length, or blank ID");
    recs[i] = ffa_record{e.data_ptr(), t.numel() ? t.data_ptr<int64_t>() : nullptr,
                         e.size(0), static_cast<int32_t>(e.size(1)),
                         static_cast<int32_t>(t.numel()), static_cast<int32_t>(blanks[i]),
                         static_cast<int32_t>(fmt)};
    lengths[i] = e.size(0);
    rec(e);
    rec(t);
  }
  const uint8_t* mask = check_mask(emission_validity, device, count, rec);
  return run_align(recs, device, mode, mask, check_inputs, stream, std::move(lengths));
}

// CPU int64 [n] view of a count vector (frames, tokens, blank IDs).
const int64_t* host_counts(const at::Tensor& t, int64_t n, const char* what) {
  TORCH_CHECK_VALUE(t.device().is_cpu() && t.scalar_type() == at::kLong && t.dim() == 1 &&
                        t.is_contiguous() && t.numel() == n,
                    what);
  return t.data_ptr<int64_t>();
}

// align_packed(Tensor emissions, Tensor frames, Tensor targets, Tensor tokens,
//              Tensor blanks, int mode, Tensor? emission_validity,
//              bool check_inputs, int fmt) -> Tensor[]
// Packed varlen form: record i is rows [sum frames[:i], +frames[i]) of a
// contiguous fp32 [N, V] matrix and tokens [sum tokens[:i], +tokens[i]) of a
// contiguous int64 vector.  One storage each, so no per-record tensors; the
// counts are CPU int64 vectors (blanks: one entry, or one per record), so no
// per-record Python objects either.
std::vector<at::Tensor> align_packed(
    const at::Tensor& emissions, const at::Tensor& frames_t, const at::Tensor& targets,
    const at::Tensor& tokens_t, const at::Tensor& blanks_t, int64_t mode,
    const std::optional<at::Tensor>& emission_validity, bool check_inputs, int64_t fmt) {
  check_mode(mode);
  const at::ScalarType dtype = format_dtype(fmt);
  const int64_t count = frames_t.numel();
  TORCH_CHECK_VALUE(count > 0 && count <= FFA_MAX_RECORDS && tokens_t.numel() == count &&
                        (blanks_t.numel() == count || blanks_t.numel() == 1),
                    "provide 1..65535 matching frame counts, token counts and blanks");
  const char* counts_msg = "frame counts, token counts and blanks must be 1-D CPU int64 vectors";
  const int64_t* frames = host_counts(frames_t, count, counts_msg);
  const int64_t* tokens = host_counts(tokens_t, count, counts_msg);
  const int64_t* blanks = host_counts(blanks_t, blanks_t.numel(), counts_msg);
  const int64_t blank_step = blanks_t.numel() == 1 ? 0 : 1;
  const auto device = emissions.device();
  TORCH_CHECK_VALUE(device.is_cuda() && targets.device() == device &&
                        emissions.scalar_type() == dtype && targets.scalar_type() == at::kLong &&
                        emissions.dim() == 2 && targets.dim() == 1 && emissions.is_contiguous() &&
                        targets.is_contiguous(),
                    format_message(fmt, true));
  const int64_t V = emissions.size(1);
  TORCH_CHECK_VALUE(V > 0 && V <= FFA_MAX_VOCAB, "unsupported vocabulary");
  c10::cuda::CUDAGuard guard(device);
  const auto stream = c10::cuda::getCurrentCUDAStream();
  StreamRecorder rec{stream};
  rec(emissions);
  rec(targets);
  thread_local std::vector<ffa_record> recs;
  recs.resize(count);
  int64_t row = 0, tok = 0;
  const auto* ebase = static_cast<const char*>(emissions.numel() ? emissions.data_ptr() : nullptr);
  const int64_t row_bytes = V * static_cast<int64_t>(emissions.element_size());
  const int64_t* tbase = targets.numel() ? targets.data_ptr<int64_t>() : nullptr;
  const int64_t rows = emissions.size(0), ntok = targets.numel();
  for (int64_t i = 0; i < count; ++i) {
    const int64_t T = frames[i], U = tokens[i], blank = blanks[i * blank_step];
    TORCH_CHECK_VALUE(T > 0 && T <= INT_MAX && U >= 0 && U <= FFA_MAX_TOKENS && blank >= 0 && blank < V,
                      "unsupported frame count, target length, or blank ID");
    TORCH_CHECK_VALUE(row + T <= rows && tok + U <= ntok,
                      "frame or token counts exceed the packed tensors");
    recs[i] = ffa_record{ebase + row * row_bytes, U ? tbase + tok : nullptr, T, static_cast<int32_t>(V),
                         static_cast<int32_t>(U), static_cast<int32_t>(blank), static_cast<int32_t>(fmt)};
    row += T;
    tok += U;
  }
  const uint8_t* mask = check_mask(emission_validity, device, count, rec);
  return std::get<0>(run_align(recs, device, mode, mask, check_inputs, stream, {}));
}

// align_stream(Tensor emissions, Tensor frames, Tensor targets, Tensor tokens,
//              Tensor blanks, int mode, bool check_inputs, int fmt, int device,
//              int copy_in, int compute, int copy_out) -> Tensor[]
// One batch of host-resident packed inputs (pinned for the copies to be
// asynchronous): host->device copies on stream `copy_in`; the align on
// `compute` once they have landed; one device->host copy of the output
// block's labels .. objective span on `copy_out` into a pinned block.
// Returns labels, scores, status, objective as views of that block.  The
// streams are torch stream ids of `device`; the caller records an event on
// `copy_out` to learn when the results are in.  Doing the whole submission
// here costs one dispatcher call instead of a dozen Python-level operations.
std::vector<at::Tensor> align_stream(const at::Tensor& emissions, const at::Tensor& frames_t,
                                     const at::Tensor& targets, const at::Tensor& tokens_t,
                                     const at::Tensor& blanks_t, int64_t mode, bool check_inputs, int64_t fmt,
                                     int64_t device_index, int64_t copy_in_id, int64_t compute_id,
                                     int64_t copy_out_id) {
  TORCH_CHECK_VALUE(emissions.device().is_cpu() && targets.device().is_cpu(),
                    "emissions and targets must be host tensors");
  TORCH_CHECK_VALUE(device_index >= 0 && device_index < 64, "device index out of range");
  const c10::Device device(c10::DeviceType::CUDA, static_cast<c10::DeviceIndex>(device_index));
  c10::cuda::CUDAGuard guard(device);
  auto stream_of = [&](int64_t id) {
    return c10::cuda::CUDAStream::unpack3(id, static_cast<c10::DeviceIndex>(device_index), c10::DeviceType::CUDA);
  };
  const c10::cuda::CUDAStream copy_in = stream_of(copy_in_id), compute = stream_of(compute_id),
                              copy_out = stream_of(copy_out_id);
  at::Tensor e, t;
  {
    c10::cuda::CUDAStreamGuard on(copy_in);
    e = at::empty(emissions.sizes(), emissions.options().device(device));
    t = at::empty(targets.sizes(), targets.options().device(device));
    e.copy_(emissions, /*non_blocking=*/true);
    t.copy_(targets, /*non_blocking=*/true);
  }
  at::cuda::CUDAEvent landed;
  landed.record(copy_in);
  landed.block(compute);
  std::vector<at::Tensor> out;
  {
    c10::cuda::CUDAStreamGuard on(compute);
    out = align_packed(e, frames_t, t, tokens_t, blanks_t, mode, std::nullopt, check_inputs, fmt);
  }
  // e and t were allocated on copy_in and are read on compute.
  c10::cuda::CUDACachingAllocator::recordStream(e.storage().data_ptr(), compute);
  c10::cuda::CUDACachingAllocator::recordStream(t.storage().data_ptr(), compute);
  at::cuda::CUDAEvent aligned;
  aligned.record(compute);
  aligned.block(copy_out);
  // labels, scores, status, objective: one allocation (OutputBlock), copied
  // back as one span.
  const at::Tensor* fields[4] = {&out[0], &out[1], &out[2], &out[3]};
  int64_t lo = INT64_MAX, hi = 0;
  for (const at::Tensor* f : fields) {
    TORCH_CHECK(f->storage().is_alias_of(out[0].storage()), "align outputs must share one allocation");
    const int64_t start = f->storage_offset() * static_cast<int64_t>(f->element_size());
    lo = std::min(lo, start);
    hi = std::max(hi, start + f->numel() * static_cast<int64_t>(f->element_size()));
  }
  c10::cuda::CUDAStreamGuard on(copy_out);
  at::Tensor span = at::empty({0}, out[0].options().dtype(at::kByte));
  span.set_(out[0].storage(), lo, {hi - lo}, {1});
  at::Tensor host = at::empty({hi - lo}, at::TensorOptions().dtype(at::kByte).pinned_memory(true));
  host.copy_(span, /*non_blocking=*/true);
  c10::cuda::CUDACachingAllocator::recordStream(out[0].storage().data_ptr(), copy_out);
  std::vector<at::Tensor> result;
  for (const at::Tensor* f : fields) {
    const int64_t start = f->storage_offset() * static_cast<int64_t>(f->element_size());
    const int64_t bytes = f->numel() * static_cast<int64_t>(f->element_size());
    result.push_back(host.narrow(0, start - lo, bytes).view(f->scalar_type()).view(f->sizes()));
  }
  return result;
}

// emission_validity(Tensor[] emissions) -> Tensor   (alignment.cu:893-917)
at::Tensor emission_validity(at::TensorList emissions) {
  const int64_t count = static_cast<int64_t>(emissions.size());
  TORCH_CHECK_VALUE(count > 0 && count <= FFA_MAX_RECORDS, "provide 1..65535 emission tensors");
  const auto device = emissions[0].device();
  const char* msg = "emissions must be contiguous CUDA float32 [T,V] with supported dimensions on one device";
  TORCH_CHECK_VALUE(device.is_cuda(), msg);
  c10::cuda::CUDAGuard guard(device);
  const auto stream = c10::cuda::getCurrentCUDAStream();
  StreamRecorder rec{stream};
  std::vector<ffa_record> recs(count);
  for (int64_t i = 0; i < count; ++i) {
    const auto& e = emissions[i];
    TORCH_CHECK_VALUE(e.device() == device && e.scalar_type() == at::kFloat && e.dim() == 2 &&
                          e.is_contiguous() && e.size(0) > 0 && e.size(0) <= INT_MAX &&
                          e.size(1) > 0 && e.size(1) <= FFA_MAX_VOCAB,
                      msg);
    recs[i] = ffa_record{e.data_ptr<float>(), nullptr, e.size(0), static_cast<int32_t>(e.size(1)), 0, 0,
                         FFA_INPUT_LOG_PROBS};
    rec(e);
  }
  ffa_sizes sizes{};
  check_status(ffa_emission_validity_query(recs.data(), count, &sizes));
  auto result = at::empty({count}, emissions[0].options().dtype(at::kBool));
  auto workspace = device_scratch(sizes.workspace_bytes);
  PinnedStaging& staging = staging_for(device.index());
  const int rc = ffa_emission_validity(recs.data(), count,
                                       reinterpret_cast<uint8_t*>(result.data_ptr<bool>()),
                                       staging.acquire(sizes.staging_bytes), sizes.staging_bytes,
                                       workspace.get(), std::max<size_t>(sizes.workspace_bytes, 256),
                                       reinterpret_cast<ffa_stream_t>(stream.stream()));
  if (rc == FFA_OK) staging.release(stream.stream());
  check_status(rc);
  return result;
}

// check_targets(Tensor[] emissions, Tensor[] targets, int[] blanks) -> Tensor
// Device int32 [B] statuses 0/3/4 (alignment.cu:852-874), nothing read back.
at::Tensor check_targets(at::TensorList emissions, at::TensorList targets, at::IntArrayRef blanks) {
  const int64_t count = static_cast<int64_t>(emissions.size());
  TORCH_CHECK_VALUE(count > 0 && count <= FFA_MAX_RECORDS &&
                        static_cast<int64_t>(targets.size()) == count &&
                        static_cast<int64_t>(blanks.size()) == count,
                    "provide 1..65535 matching emissions and targets");
  const auto device = emissions[0].device();
  const char* msg = "inputs must be contiguous CUDA float32 or bfloat16 [T,V] and int64 [U] on one device";
  TORCH_CHECK_VALUE(device.is_cuda(), msg);
  c10::cuda::CUDAGuard guard(device);
  const auto stream = c10::cuda::getCurrentCUDAStream();
  StreamRecorder rec{stream};
  std::vector<ffa_record> recs(count);
  for (int64_t i = 0; i < count; ++i) {
    const auto& e = emissions[i];
    const auto& t = targets[i];
    TORCH_CHECK_VALUE(e.device() == device && t.device() == device &&
                          (e.scalar_type() == at::kFloat || e.scalar_type() == at::kBFloat16) &&
                          t.scalar_type() == at::kLong && e.dim() == 2 && t.dim() == 1 && e.is_contiguous() &&
                          t.is_contiguous(),
                      msg);
    TORCH_CHECK_VALUE(e.size(0) > 0 && e.size(0) <= INT_MAX && e.size(1) > 0 &&
                          e.size(1) <= FFA_MAX_VOCAB && t.numel() <= FFA_MAX_TOKENS && blanks[i] >= 0 &&
                          blanks[i] < e.size(1),
                      "unsupported frame count, vocabulary, target length, or blank ID");
    // Only the shapes and targets are read: logits check as log-probabilities do.
    recs[i] = ffa_record{e.data_ptr(), t.numel() ? t.data_ptr<int64_t>() : nullptr,
                         e.size(0), static_cast<int32_t>(e.size(1)),
                         static_cast<int32_t>(t.numel()), static_cast<int32_t>(blanks[i]),
                         e.scalar_type() == at::kBFloat16 ? FFA_INPUT_LOGITS_BF16 : FFA_INPUT_LOG_PROBS};
    rec(t);
  }
  ffa_sizes sizes{};
  check_status(ffa_check_targets_query(recs.data(), count, &sizes));
  auto status = at::empty({count}, emissions[0].options().dtype(at::kInt));
  auto workspace = device_scratch(sizes.workspace_bytes);
  PinnedStaging& staging = staging_for(device.index());
  const int rc = ffa_check_targets(recs.data(), count, status.data_ptr<int32_t>(),
                                   staging.acquire(sizes.staging_bytes), sizes.staging_bytes,
                                   workspace.get(), std::max<size_t>(sizes.workspace_bytes, 256),
                                   reinterpret_cast<ffa_stream_t>(stream.stream()));
  if (rc == FFA_OK) staging.release(stream.stream());
  check_status(rc);
  return status;
}

// token_spans(Tensor labels, Tensor frames, Tensor tokens, Tensor blanks) -> Tensor
// labels: CUDA int64 [sum frames] (an align output); frames, tokens: CPU int64
// [B]; blanks: CPU int64 [1] or [B].  Returns CUDA int64 [sum tokens, 2].
at::Tensor token_spans(const at::Tensor& labels, const at::Tensor& frames_t, const at::Tensor& tokens_t,
                       const at::Tensor& blanks_t) {
  const int64_t count = frames_t.numel();
  TORCH_CHECK_VALUE(count > 0 && count <= FFA_MAX_RECORDS && tokens_t.numel() == count &&
                        (blanks_t.numel() == 1 || blanks_t.numel() == count),
                    "provide 1..65535 matching frame counts, token counts and blanks");
  const char* counts_msg = "frame counts, token counts and blanks must be 1-D CPU int64 vectors";
  const int64_t* frames = host_counts(frames_t, count, counts_msg);
  const int64_t* tokens64 = host_counts(tokens_t, count, counts_msg);
  const int64_t* blanks64 = host_counts(blanks_t, blanks_t.numel(), counts_msg);
  TORCH_CHECK_VALUE(labels.device().is_cuda() && labels.scalar_type() == at::kLong && labels.dim() == 1 &&
                        labels.is_contiguous(),
                    "labels must be a contiguous CUDA int64 vector");
  std::vector<int32_t> tokens(count), blanks(count);
  int64_t frames_total = 0, tokens_total = 0;
  for (int64_t i = 0; i < count; ++i) {
    TORCH_CHECK_VALUE(tokens64[i] >= 0 && tokens64[i] <= FFA_MAX_TOKENS, "unsupported token count");
    const int64_t b = blanks64[blanks_t.numel() == 1 ? 0 : i];
    TORCH_CHECK_VALUE(b >= 0 && b <= INT_MAX, "unsupported blank ID");
    tokens[i] = static_cast<int32_t>(tokens64[i]);
    blanks[i] = static_cast<int32_t>(b);
    frames_total += frames[i];
    tokens_total += tokens64[i];
  }
  TORCH_CHECK_VALUE(frames_total == labels.numel(), "frame counts must add up to the labels' length");
  const auto device = labels.device();
  c10::cuda::CUDAGuard guard(device);
  const auto stream = c10::cuda::getCurrentCUDAStream();
  StreamRecorder rec{stream};
  rec(labels);
  ffa_sizes sizes{};
  check_status(ffa_token_spans_query(frames, tokens.data(), count, &sizes));
  auto spans = at::empty({tokens_total, 2}, labels.options());
  auto workspace = device_scratch(sizes.workspace_bytes);
  PinnedStaging& staging = staging_for(device.index());
  const int rc = ffa_token_spans(labels.data_ptr<int64_t>(), frames, tokens.data(), blanks.data(), count,
                                 tokens_total ? spans.data_ptr<int64_t>() : nullptr,
                                 staging.acquire(sizes.staging_bytes), sizes.staging_bytes, workspace.get(),
                                 std::max<size_t>(sizes.workspace_bytes, 256),
                                 reinterpret_cast<ffa_stream_t>(stream.stream()));
  if (rc == FFA_OK) staging.release(stream.stream());
  check_status(rc);
  return spans;
}

// row_logsumexp(Tensor[] logits) -> Tensor
// CUDA float32 [sum T]: each row's log-sum-exp as ffa_align subtracts it
// from logits (fp32 or bf16, one dtype for the list).
at::Tensor row_logsumexp(at::TensorList logits) {
  const int64_t count = static_cast<int64_t>(logits.size());
  TORCH_CHECK_VALUE(count > 0 && count <= FFA_MAX_RECORDS, "provide 1..65535 logits tensors");
  const auto device = logits[0].device();
  const at::ScalarType dtype = logits[0].scalar_type();
  const char* msg = "logits must be contiguous CUDA float32 or bfloat16 [T,V] tensors of one dtype on one device";
  TORCH_CHECK_VALUE(device.is_cuda() && (dtype == at::kFloat || dtype == at::kBFloat16), msg);
  const int32_t fmt = dtype == at::kBFloat16 ? FFA_INPUT_LOGITS_BF16 : FFA_INPUT_LOGITS_F32;
  c10::cuda::CUDAGuard guard(device);
  const auto stream = c10::cuda::getCurrentCUDAStream();
  StreamRecorder rec{stream};
  std::vector<ffa_record> recs(count);
  int64_t rows = 0;
  for (int64_t i = 0; i < count; ++i) {
    const auto& e = logits[i];
    TORCH_CHECK_VALUE(e.device() == device && e.scalar_type() == dtype && e.dim() == 2 && e.is_contiguous() &&
                          e.size(0) > 0 && e.size(0) <= INT_MAX && e.size(1) > 0 && e.size(1) <= FFA_MAX_VOCAB,
                      msg);
    recs[i] = ffa_record{e.data_ptr(), nullptr, e.size(0), static_cast<int32_t>(e.size(1)), 0, 0, fmt};
    rows += e.size(0);
    rec(e);
  }
  ffa_sizes sizes{};
  check_status(ffa_row_logsumexp_query(recs.data(), count, &sizes));
  auto z = at::empty({rows}, logits[0].options().dtype(at::kFloat));
  auto workspace = device_scratch(sizes.workspace_bytes);
  PinnedStaging& staging = staging_for(device.index());
  const int rc = ffa_row_logsumexp(recs.data(), count, z.data_ptr<float>(), staging.acquire(sizes.staging_bytes),
                                   sizes.staging_bytes, workspace.get(), std::max<size_t>(sizes.workspace_bytes, 256),
                                   reinterpret_cast<ffa_stream_t>(stream.stream()));
  if (rc == FFA_OK) staging.release(stream.stream());
  check_status(rc);
  return z;
}

}  // namespace

TORCH_LIBRARY(ffa_b200, m) {
  m.def("align(Tensor[] emissions, Tensor[] targets, int[] blanks, int mode, "
        "Tensor? emission_validity=None, bool check_inputs=True, int fmt=0) -> (Tensor[], int[])");
  m.def("align_packed(Tensor emissions, Tensor frames, Tensor targets, Tensor tokens, Tensor blanks, "
        "int mode, Tensor? emission_validity=None, bool check_inputs=True, int fmt=0) -> Tensor[]");
  m.def("row_logsumexp(Tensor[] logits) -> Tensor");
  m.def("align_stream(Tensor emissions, Tensor frames, Tensor targets, Tensor tokens, Tensor blanks, int mode, "
        "bool check_inputs, int fmt, int device, int copy_in, int compute, int copy_out) -> Tensor[]");
  m.def("emission_validity(Tensor[] emissions) -> Tensor");
  m.def("check_targets(Tensor[] emissions, Tensor[] targets, int[] blanks) -> Tensor");
  m.def("token_spans(Tensor labels, Tensor frames, Tensor tokens, Tensor blanks) -> Tensor");
}

TORCH_LIBRARY_IMPL(ffa_b200, CUDA, m) {
  m.impl("align", &align);
  m.impl("align_packed", &align_packed);
  m.impl("emission_validity", &emission_validity);
  m.impl("check_targets", &check_targets);
  m.impl("token_spans", &token_spans);
  m.impl("row_logsumexp", &row_logsumexp);
}

// align_stream takes host tensors and stream ids: registered for the CPU
// dispatch key (its inputs' device), it runs on the CUDA device it is given.
TORCH_LIBRARY_IMPL(ffa_b200, CPU, m) {
  m.impl("align_stream", &align_stream);
}
