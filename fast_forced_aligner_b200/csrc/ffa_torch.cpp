// ffa_torch.cpp -- thin PyTorch operator layer over the C ABI (libffa_b200.so).
//
// Registers torch.ops.ffa_b200.{align, align_packed, emission_validity}.  It
// mirrors the reference's op layer (alignment.cu:893-1061,
// TORCH_LIBRARY at alignment.cu:1064-1070): tensor metadata checks, stream
// lifetime protection (recordStream on borrowed inputs), output allocation
// from the caching allocator, and a pinned staging buffer whose reuse is
// fenced with the host allocator's stream event.  Everything below the
// ffa_* calls is plain pointers and sizes.
#include <ATen/ATen.h>
#include <ATen/core/CachingHostAllocator.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <climits>
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

at::Tensor pinned_staging(size_t bytes) {
  return at::empty({static_cast<int64_t>(std::max<size_t>(bytes, 1))},
                   at::TensorOptions().dtype(at::kByte).device(at::kCPU).pinned_memory(true));
}

void fence_staging(const at::Tensor& staging, c10::cuda::CUDAStream stream) {
  at::getHostAllocator(at::kCUDA)->record_event(
      staging.data_ptr(), staging.storage().data_ptr().get_context(), stream.unwrap());
}

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
  const int cmode = mode == 0 ? FFA_MODE_CONVENTIONAL : FFA_MODE_OPTIMIZED;
  const int flags = check_inputs ? FFA_FLAG_CHECK_INPUTS : 0;
  ffa_sizes sizes{};
  check_status(ffa_align_query(recs.data(), count, cmode, flags, &sizes));

  // One caching-allocator block per output (cheaper than carving typed views
  // out of one block, which costs several dispatcher calls per view).
  const int64_t N = sizes.total_frames;
  int64_t max_frames = 0;
  for (const auto& r : recs) max_frames = std::max(max_frames, r.frames);
  const bool reuse = cmode == FFA_MODE_OPTIMIZED && max_frames >= 2048;
  const auto opts = at::TensorOptions().device(device);
  auto labels = at::empty({N}, opts.dtype(at::kLong));
  auto scores = at::empty({N}, opts.dtype(at::kFloat));
  auto status = at::empty({count}, opts.dtype(at::kInt));
  auto objective = at::empty({count}, opts.dtype(at::kFloat));
  auto stitched = at::empty({count}, opts.dtype(at::kInt));
  auto passes = at::empty({count}, opts.dtype(at::kInt));
  auto repaired = at::empty({count}, opts.dtype(at::kLong));
  auto shortcut = at::empty({count, 3}, opts.dtype(at::kLong));
  auto routing = at::empty({count, 3}, opts.dtype(at::kInt));
  auto reuse_stats = at::empty({reuse ? count : 0, 4}, opts.dtype(at::kLong));

  auto staging = pinned_staging(sizes.staging_bytes);
  auto workspace = at::empty({static_cast<int64_t>(std::max<size_t>(sizes.workspace_bytes, 256))},
                             opts.dtype(at::kByte));
  ffa_outputs out{labels.data_ptr<int64_t>(), scores.data_ptr<float>(), status.data_ptr<int32_t>(),
                  objective.data_ptr<float>(), stitched.data_ptr<int32_t>(),
                  passes.data_ptr<int32_t>(), repaired.data_ptr<int64_t>(),
                  shortcut.data_ptr<int64_t>(), routing.data_ptr<int32_t>(),
                  reuse ? reuse_stats.data_ptr<int64_t>() : nullptr};
  const int rc = ffa_align(recs.data(), count, cmode, flags, mask, &out, staging.data_ptr(),
                           sizes.staging_bytes, workspace.data_ptr(),
                           static_cast<size_t>(workspace.numel()),
                           reinterpret_cast<ffa_stream_t>(stream.stream()));
  fence_staging(staging, stream);
  check_status(rc);
  return {{labels, scores, status, objective, stitched, passes, repaired, shortcut, routing,
           reuse_stats},
          std::move(lengths)};
}

void check_mode(int64_t mode) {
  TORCH_CHECK_VALUE(mode == 0 || mode == 1, "mode must be 'optimized' or 'conventional'");
}

// align(Tensor[] emissions, Tensor[] targets, int[] blanks, int mode,
//       Tensor? emission_validity, bool check_inputs) -> (Tensor[], int[])
std::tuple<std::vector<at::Tensor>, std::vector<int64_t>> align(
    at::TensorList emissions, at::TensorList targets, at::IntArrayRef blanks, int64_t mode,
    const std::optional<at::Tensor>& emission_validity, bool check_inputs) {
  check_mode(mode);
  const int64_t count = static_cast<int64_t>(emissions.size());
  TORCH_CHECK_VALUE(count > 0 && count <= FFA_MAX_RECORDS &&
                        static_cast<int64_t>(targets.size()) == count &&
                        static_cast<int64_t>(blanks.size()) == count,
                    "provide 1..65535 matching emissions and targets");
  const auto device = emissions[0].device();
  TORCH_CHECK_VALUE(device.is_cuda(), "inputs must be contiguous CUDA float32 [T,V] and int64 [U] on one device");
  c10::cuda::CUDAGuard guard(device);
  const auto stream = c10::cuda::getCurrentCUDAStream();
  StreamRecorder rec{stream};
  std::vector<ffa_record> recs(count);
  std::vector<int64_t> lengths(count);
  for (int64_t i = 0; i < count; ++i) {
    const auto& e = emissions[i];
    const auto& t = targets[i];
    TORCH_CHECK_VALUE(e.device() == device && t.device() == device &&
                          e.scalar_type() == at::kFloat && t.scalar_type() == at::kLong &&
                          e.dim() == 2 && t.dim() == 1 && e.is_contiguous() && t.is_contiguous(),
                      "inputs must be contiguous CUDA float32 [T,V] and int64 [U] on one device");
    TORCH_CHECK_VALUE(e.size(0) > 0 && e.size(0) <= INT_MAX && e.size(1) > 0 &&
                          e.size(1) <= FFA_MAX_VOCAB && t.numel() <= 2047 && blanks[i] >= 0 &&
                          blanks[i] < e.size(1),
                      "unsupported frame count, vocabulary, target length, or blank ID");
    recs[i] = ffa_record{e.data_ptr<float>(), t.numel() ? t.data_ptr<int64_t>() : nullptr,
                         e.size(0), static_cast<int32_t>(e.size(1)),
                         static_cast<int32_t>(t.numel()), static_cast<int32_t>(blanks[i]), 0};
    lengths[i] = e.size(0);
    rec(e);
    rec(t);
  }
  const uint8_t* mask = check_mask(emission_validity, device, count, rec);
  return run_align(recs, device, mode, mask, check_inputs, stream, std::move(lengths));
}

// align_packed(Tensor emissions, int[] frames, Tensor targets, int[] tokens,
//              int[] blanks, int mode, Tensor? emission_validity,
//              bool check_inputs) -> (Tensor[], int[])
// Packed varlen form: record i is rows [sum frames[:i], +frames[i]) of a
// contiguous fp32 [N, V] matrix and tokens [sum tokens[:i], +tokens[i]) of a
// contiguous int64 vector.  One storage each, so no per-record tensors.
std::tuple<std::vector<at::Tensor>, std::vector<int64_t>> align_packed(
    const at::Tensor& emissions, at::IntArrayRef frames, const at::Tensor& targets,
    at::IntArrayRef tokens, at::IntArrayRef blanks, int64_t mode,
    const std::optional<at::Tensor>& emission_validity, bool check_inputs) {
  check_mode(mode);
  const int64_t count = static_cast<int64_t>(frames.size());
  TORCH_CHECK_VALUE(count > 0 && count <= FFA_MAX_RECORDS &&
                        static_cast<int64_t>(tokens.size()) == count &&
                        static_cast<int64_t>(blanks.size()) == count,
                    "provide 1..65535 matching frame counts, token counts and blanks");
  const auto device = emissions.device();
  TORCH_CHECK_VALUE(device.is_cuda() && targets.device() == device &&
                        emissions.scalar_type() == at::kFloat && targets.scalar_type() == at::kLong &&
                        emissions.dim() == 2 && targets.dim() == 1 && emissions.is_contiguous() &&
                        targets.is_contiguous(),
                    "inputs must be contiguous CUDA float32 [N,V] and int64 [M] on one device");
  const int64_t V = emissions.size(1);
  TORCH_CHECK_VALUE(V > 0 && V <= FFA_MAX_VOCAB, "unsupported vocabulary");
  c10::cuda::CUDAGuard guard(device);
  const auto stream = c10::cuda::getCurrentCUDAStream();
  StreamRecorder rec{stream};
  rec(emissions);
  rec(targets);
  std::vector<ffa_record> recs(count);
  std::vector<int64_t> lengths(frames.begin(), frames.end());
  int64_t row = 0, tok = 0;
  const float* ebase = emissions.numel() ? emissions.data_ptr<float>() : nullptr;
  const int64_t* tbase = targets.numel() ? targets.data_ptr<int64_t>() : nullptr;
  for (int64_t i = 0; i < count; ++i) {
    TORCH_CHECK_VALUE(frames[i] > 0 && frames[i] <= INT_MAX && tokens[i] >= 0 && tokens[i] <= 2047 &&
                          blanks[i] >= 0 && blanks[i] < V,
                      "unsupported frame count, target length, or blank ID");
    TORCH_CHECK_VALUE(row + frames[i] <= emissions.size(0) && tok + tokens[i] <= targets.numel(),
                      "frame or token counts exceed the packed tensors");
    recs[i] = ffa_record{ebase + row * V, tokens[i] ? tbase + tok : nullptr, frames[i],
                         static_cast<int32_t>(V), static_cast<int32_t>(tokens[i]),
                         static_cast<int32_t>(blanks[i]), 0};
    row += frames[i];
    tok += tokens[i];
  }
  const uint8_t* mask = check_mask(emission_validity, device, count, rec);
  return run_align(recs, device, mode, mask, check_inputs, stream, std::move(lengths));
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
    recs[i] = ffa_record{e.data_ptr<float>(), nullptr, e.size(0), static_cast<int32_t>(e.size(1)), 0, 0, 0};
    rec(e);
  }
  ffa_sizes sizes{};
  check_status(ffa_emission_validity_query(recs.data(), count, &sizes));
  auto result = at::empty({count}, emissions[0].options().dtype(at::kBool));
  auto staging = pinned_staging(sizes.staging_bytes);
  auto workspace = at::empty({static_cast<int64_t>(std::max<size_t>(sizes.workspace_bytes, 256))},
                             emissions[0].options().dtype(at::kByte));
  const int rc = ffa_emission_validity(recs.data(), count,
                                       reinterpret_cast<uint8_t*>(result.data_ptr<bool>()),
                                       staging.data_ptr(), sizes.staging_bytes, workspace.data_ptr(),
                                       static_cast<size_t>(workspace.numel()),
                                       reinterpret_cast<ffa_stream_t>(stream.stream()));
  fence_staging(staging, stream);
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
  const char* msg = "inputs must be contiguous CUDA float32 [T,V] and int64 [U] on one device";
  TORCH_CHECK_VALUE(device.is_cuda(), msg);
  c10::cuda::CUDAGuard guard(device);
  const auto stream = c10::cuda::getCurrentCUDAStream();
  StreamRecorder rec{stream};
  std::vector<ffa_record> recs(count);
  for (int64_t i = 0; i < count; ++i) {
    const auto& e = emissions[i];
    const auto& t = targets[i];
    TORCH_CHECK_VALUE(e.device() == device && t.device() == device &&
                          e.scalar_type() == at::kFloat && t.scalar_type() == at::kLong &&
                          e.dim() == 2 && t.dim() == 1 && e.is_contiguous() && t.is_contiguous(),
                      msg);
    TORCH_CHECK_VALUE(e.size(0) > 0 && e.size(0) <= INT_MAX && e.size(1) > 0 &&
                          e.size(1) <= FFA_MAX_VOCAB && t.numel() <= 2047 && blanks[i] >= 0 &&
                          blanks[i] < e.size(1),
                      "unsupported frame count, vocabulary, target length, or blank ID");
    recs[i] = ffa_record{e.data_ptr<float>(), t.numel() ? t.data_ptr<int64_t>() : nullptr,
                         e.size(0), static_cast<int32_t>(e.size(1)),
                         static_cast<int32_t>(t.numel()), static_cast<int32_t>(blanks[i]), 0};
    rec(t);
  }
  ffa_sizes sizes{};
  check_status(ffa_check_targets_query(recs.data(), count, &sizes));
  auto status = at::empty({count}, emissions[0].options().dtype(at::kInt));
  auto staging = pinned_staging(sizes.staging_bytes);
  auto workspace = at::empty({static_cast<int64_t>(std::max<size_t>(sizes.workspace_bytes, 256))},
                             emissions[0].options().dtype(at::kByte));
  const int rc = ffa_check_targets(recs.data(), count, status.data_ptr<int32_t>(), staging.data_ptr(),
                                   sizes.staging_bytes, workspace.data_ptr(),
                                   static_cast<size_t>(workspace.numel()),
                                   reinterpret_cast<ffa_stream_t>(stream.stream()));
  fence_staging(staging, stream);
  check_status(rc);
  return status;
}

}  // namespace

TORCH_LIBRARY(ffa_b200, m) {
  m.def("align(Tensor[] emissions, Tensor[] targets, int[] blanks, int mode, "
        "Tensor? emission_validity=None, bool check_inputs=True) -> (Tensor[], int[])");
  m.def("align_packed(Tensor emissions, int[] frames, Tensor targets, int[] tokens, int[] blanks, "
        "int mode, Tensor? emission_validity=None, bool check_inputs=True) -> (Tensor[], int[])");
  m.def("emission_validity(Tensor[] emissions) -> Tensor");
  m.def("check_targets(Tensor[] emissions, Tensor[] targets, int[] blanks) -> Tensor");
}

TORCH_LIBRARY_IMPL(ffa_b200, CUDA, m) {
  m.impl("align", &align);
  m.impl("align_packed", &align_packed);
  m.impl("emission_validity", &emission_validity);
  m.impl("check_targets", &check_targets);
}
