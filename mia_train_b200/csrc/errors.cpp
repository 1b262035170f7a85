#include "errors.h"

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>
#include <unordered_map>

namespace mia {

namespace {
std::mutex g_lock;
// Never destroyed: the tensors must not be freed after the CUDA context is torn down at exit.
std::unordered_map<int, at::Tensor>& g_words = *new std::unordered_map<int, at::Tensor>();
}  // namespace

int* error_word(int device) {
  std::lock_guard<std::mutex> guard(g_lock);
  auto it = g_words.find(device);
  if (it == g_words.end()) {
    c10::cuda::CUDAGuard dev(device);
    auto t = at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, device));
    it = g_words.emplace(device, t).first;
  }
  return it->second.data_ptr<int>();
}

int64_t read_and_clear_errors(int64_t device) {
  int* word = error_word((int)device);
  c10::cuda::CUDAGuard dev((int)device);
  int host = 0;
  C10_CUDA_CHECK(cudaMemcpy(&host, word, sizeof(int), cudaMemcpyDeviceToHost));
  if (host != 0) C10_CUDA_CHECK(cudaMemset(word, 0, sizeof(int)));
  return host;
}

}  // namespace mia
