// C++ API checks, built without gtest (none is available offline) and run by
// tests/test_cpp_api_gpu.py.  Mirrors the reference's C++ tests:
//  * Tensor semantics of test/tensor_test.cpp: zero-filled allocation,
//    metadata-only resize, no reallocation when shrinking, reallocation when
//    growing, host <-> device round trip, shared ownership on copy;
//  * the attention smoke run of test/cuda/mha_attention_test.cpp (h=4,
//    kv_h=2, S=256, D=128, fp16, zero inputs), now with its output checked;
//  * a known answer: with q = 0 every visible key gets the same weight, so
//    causal O[i] is the mean of V[0..i] (per kv head), computed here on the host;
//  * the operator registry (include/llmx/ops.h): test/ops_test.cpp:8-31's
//    fp16 [1, 2, 3, 4] -> to_fp32 known answer, to_fp16 / to_bf16 (the
//    reference's to_fp16 cannot run: it looks up "tto_fp16_op"), a dtype
//    change that must reallocate, and "attention_haft_op" against the direct
//    call, bit for bit.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <vector>

#include "llmx/cuda/attention/attention_api.h"
#include "llmx/ops.h"
#include "llmx/tensor.h"

using namespace llmx;

static int g_fail = 0;
#define EXPECT(cond)                                                   \
  do {                                                                 \
    if (!(cond)) {                                                     \
      std::fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond); \
      ++g_fail;                                                        \
    }                                                                  \
  } while (0)

static void tensor_semantics() {
  Device cpu(DeviceType::kCPU), gpu(DeviceType::kCUDA, 0);
  Tensor t({2, 3, 4}, ScalarType::kFP32, cpu);
  EXPECT(!t.is_valid());  // construction sets metadata only (tensor_test.cpp:18-28)
  t.allocate();
  EXPECT(t.is_valid());
  EXPECT(t.numel() == 24 && t.capacity() == 24 && t.contiguous());
  EXPECT(llmx_mem_info(t.data_ptr()).has_value() && llmx_mem_info(t.data_ptr())->nbytes == 96);
  EXPECT(t.stride(0) == 12 && t.stride(1) == 4 && t.stride(2) == 1 && t.count(1) == 12);
  const float *p = t.const_data_ptr<float>();
  bool zero = true;
  for (int i = 0; i < 24; ++i) zero = zero && p[i] == 0.f;
  EXPECT(zero);
  void *before = t.data_ptr();
  t.resize({4, 3});  // metadata only
  EXPECT(t.data_ptr() == before && t.numel() == 12 && t.capacity() == 24);
  t.allocate();  // shrinking: keeps the storage
  EXPECT(t.data_ptr() == before);
  t.resize({8, 8});
  t.allocate();  // growing: new storage
  EXPECT(t.capacity() == 64);
  for (int i = 0; i < 64; ++i) t.data_ptr<float>()[i] = float(i);
  t.to_device(gpu);
  EXPECT(t.device() == gpu);
  t.to_device(cpu);
  bool same = true;
  for (int i = 0; i < 64; ++i) same = same && t.const_data_ptr<float>()[i] == float(i);
  EXPECT(same);
  Tensor u = t;  // shares storage
  EXPECT(u.data_ptr() == t.data_ptr() && t.data().use_count() == 2);
}

template <typename T>
static std::vector<float> to_float(const std::vector<T> &v) {
  std::vector<float> f(v.size());
  for (size_t i = 0; i < v.size(); ++i) {
    if constexpr (std::is_same<T, __half>::value)
      f[i] = __half2float(v[i]);
    else
      f[i] = __bfloat162float(v[i]);
  }
  return f;
}

static void smoke_zero_inputs() {
  // test/cuda/mha_attention_test.cpp: all-zero q/k/v, causal, no ALiBi.
  const int S = 256, H = 4, Hkv = 2, D = 128;
  Device gpu(DeviceType::kCUDA, 0);
  Tensor q({S, H, D}, ScalarType::kFP16, cuda0), k({S, Hkv, D}, ScalarType::kFP16, cuda0),
      v({S, Hkv, D}, ScalarType::kFP16, cuda0), o({S, H, D}, ScalarType::kFP16, cuda0);
  for (Tensor *t : {&q, &k, &v, &o}) t->allocate();
  llmx_single_mha_attention(o, q, k, v, std::nullopt, 1.0f / std::sqrt(float(D)));
  EXPECT(cudaDeviceSynchronize() == cudaSuccess);
  std::vector<__half> h(o.numel());
  llmx_copy(gpu, Device(DeviceType::kCPU), o.const_data_ptr(), h.data(), o.nbytes());
  bool zero = true;
  for (auto x : to_float(h)) zero = zero && x == 0.f;
  EXPECT(zero);
}

static void known_answer_uniform_weights() {
  const int S = 200, H = 4, Hkv = 2, D = 64;
  Device gpu(DeviceType::kCUDA, 0), cpu(DeviceType::kCPU);
  std::vector<__nv_bfloat16> hq(S * H * D, __float2bfloat16(0.f)), hk(S * Hkv * D), hv(S * Hkv * D);
  unsigned s = 12345u;
  auto rnd = [&] {
    s = s * 1664525u + 1013904223u;
    return float((s >> 8) & 0xffff) / 65536.f - 0.5f;
  };
  for (auto &x : hk) x = __float2bfloat16(rnd());
  for (auto &x : hv) x = __float2bfloat16(rnd());
  Tensor q({S, H, D}, ScalarType::kBF16, gpu), k({S, Hkv, D}, ScalarType::kBF16, gpu),
      v({S, Hkv, D}, ScalarType::kBF16, gpu), o({S, H, D}, ScalarType::kBF16, gpu);
  for (Tensor *t : {&q, &k, &v, &o}) t->allocate();
  llmx_copy(cpu, gpu, hq.data(), q.data_ptr(), q.nbytes());
  llmx_copy(cpu, gpu, hk.data(), k.data_ptr(), k.nbytes());
  llmx_copy(cpu, gpu, hv.data(), v.data_ptr(), v.nbytes());
  llmx_single_mha_attention(o, q, k, v, std::nullopt, 0.125f);
  EXPECT(cudaDeviceSynchronize() == cudaSuccess);
  std::vector<__nv_bfloat16> ho(o.numel());
  llmx_copy(gpu, cpu, o.const_data_ptr(), ho.data(), o.nbytes());
  const std::vector<float> fo = to_float(ho), fv = to_float(hv);
  double max_err = 0;
  for (int h = 0; h < H; ++h) {
    const int kvh = h / (H / Hkv);
    for (int d = 0; d < D; ++d) {
      double run = 0;
      for (int i = 0; i < S; ++i) {
        run += fv[(i * Hkv + kvh) * D + d];
        const double want = run / (i + 1);
        max_err = std::fmax(max_err, std::fabs(want - fo[(i * H + h) * D + d]));
      }
    }
  }
  std::printf("known answer max error %.3e\n", max_err);
  EXPECT(max_err < 1e-2);
}

static void argument_errors_throw() {
  Device gpu(DeviceType::kCUDA, 0);
  Tensor q({16, 4, 64}, ScalarType::kFP16, gpu), k({16, 3, 64}, ScalarType::kFP16, gpu),
      v({16, 3, 64}, ScalarType::kFP16, gpu), o({16, 4, 64}, ScalarType::kFP16, gpu);
  for (Tensor *t : {&q, &k, &v, &o}) t->allocate();
  bool threw = false;
  try {
    llmx_single_mha_attention(o, q, k, v, std::nullopt, 0.125f);  // 4 heads over 3 kv heads
  } catch (const std::runtime_error &) {
    threw = true;
  }
  EXPECT(threw);
}

static void registry_conversions() {
  Device cpu(DeviceType::kCPU), gpu(DeviceType::kCUDA, 0);
  // ops_test.cpp: fp16 [1, 2, 3, 4] -> fp32.  The input starts on the host;
  // the executor moves it to the device.
  Tensor input({4}, ScalarType::kFP16, cpu);
  input.allocate();
  for (int i = 0; i < 4; ++i) input.data_ptr<__half>()[i] = __float2half(float(i + 1));
  Tensor output;
  to_fp32(output, input);
  EXPECT(cudaDeviceSynchronize() == cudaSuccess);
  EXPECT(output.is_valid() && output.dtype() == ScalarType::kFP32);
  EXPECT(output.dims() == std::vector<int>{4} && output.device() == gpu);
  EXPECT(input.device() == gpu);
  std::vector<float> f(4);
  llmx_copy(gpu, cpu, output.const_data_ptr(), f.data(), 16);
  for (int i = 0; i < 4; ++i) EXPECT(f[i] == float(i + 1));

  // fp32 -> fp16 / bf16 of values that need rounding, 1000 + 3 elements so
  // both the vector body and the tail run; checked against the host casts.
  const int n = 1003;
  Tensor src({n}, ScalarType::kFP32, cpu);
  src.allocate();
  for (int i = 0; i < n; ++i) src.data_ptr<float>()[i] = (i - 500) * 0.0123457f + 1e-4f * (i % 7);
  std::vector<float> host(src.const_data_ptr<float>(), src.const_data_ptr<float>() + n);
  Tensor h16, b16;
  to_fp16(h16, src);
  to_bf16(b16, src);
  EXPECT(cudaDeviceSynchronize() == cudaSuccess);
  std::vector<__half> gh(n);
  std::vector<__nv_bfloat16> gb(n);
  llmx_copy(gpu, cpu, h16.const_data_ptr(), gh.data(), n * 2);
  llmx_copy(gpu, cpu, b16.const_data_ptr(), gb.data(), n * 2);
  int bad = 0;
  for (int i = 0; i < n; ++i) {
    const __half eh = __float2half_rn(host[i]);
    const __nv_bfloat16 eb = __float2bfloat16_rn(host[i]);
    bad += std::memcmp(&eh, &gh[i], 2) != 0;
    bad += std::memcmp(&eb, &gb[i], 2) != 0;
  }
  EXPECT(bad == 0);

  // An output reused at a wider dtype must get new storage.
  Tensor out2;
  to_fp16(out2, src);
  const size_t narrow = out2.nbytes();
  to_fp32(out2, h16);
  EXPECT(out2.nbytes() >= size_t(n) * 4 && out2.nbytes() > narrow);
  EXPECT(cudaDeviceSynchronize() == cudaSuccess);

  bool threw = false;
  try {
    get_op_executor()->run("tto_fp16_op", {{"input", &src}, {"output", &out2}}, {});
  } catch (const std::runtime_error &) {
    threw = true;
  }
  EXPECT(threw);
}

static void registry_attention_matches_direct_call() {
  const int S = 300, H = 8, Hkv = 2, D = 128;
  Device gpu(DeviceType::kCUDA, 0), cpu(DeviceType::kCPU);
  std::vector<__half> hq(S * H * D), hk(S * Hkv * D), hv(S * Hkv * D);
  unsigned s = 777u;
  auto rnd = [&] {
    s = s * 1664525u + 1013904223u;
    return float((s >> 8) & 0xffff) / 32768.f - 1.f;
  };
  for (auto &x : hq) x = __float2half(rnd());
  for (auto &x : hk) x = __float2half(rnd());
  for (auto &x : hv) x = __float2half(rnd());
  Tensor q({S, H, D}, ScalarType::kFP16, gpu), k({S, Hkv, D}, ScalarType::kFP16, gpu),
      v({S, Hkv, D}, ScalarType::kFP16, gpu), direct({S, H, D}, ScalarType::kFP16, gpu);
  for (Tensor *t : {&q, &k, &v, &direct}) t->allocate();
  llmx_copy(cpu, gpu, hq.data(), q.data_ptr(), q.nbytes());
  llmx_copy(cpu, gpu, hk.data(), k.data_ptr(), k.nbytes());
  llmx_copy(cpu, gpu, hv.data(), v.data_ptr(), v.nbytes());
  std::vector<float> hs(H);
  for (int h = 0; h < H; ++h) hs[h] = std::exp2(-8.f * (h + 1) / H);
  Tensor slopes_cpu(hs.data(), {H}, ScalarType::kFP32, cpu);
  Tensor slopes({H}, ScalarType::kFP32, gpu);
  slopes.allocate();
  llmx_copy(cpu, gpu, hs.data(), slopes.data_ptr(), slopes.nbytes());
  const float scale = 1.f / std::sqrt(float(D));
  llmx_single_mha_attention(direct, q, k, v, slopes, scale, 100, 0.f);
  Tensor via_registry;
  Parameters params{{"alibi_slopes", std::optional<Tensor>(slopes_cpu)},  // host slopes are moved
                    {"sm_scale", scale},
                    {"sliding_window", 100},
                    {"logits_soft_cap", 0.f}};
  get_op_executor()->run("attention_haft_op",
                         {{"query", &q}, {"key", &k}, {"value", &v}, {"output", &via_registry}}, params);
  Tensor via_helper;
  attention(via_helper, q, k, v, slopes, scale, 100, 0.f);
  EXPECT(cudaDeviceSynchronize() == cudaSuccess);
  EXPECT(via_registry.dims() == q.dims() && via_registry.dtype() == ScalarType::kFP16);
  std::vector<__half> a(direct.numel()), b(direct.numel()), c(direct.numel());
  llmx_copy(gpu, cpu, direct.const_data_ptr(), a.data(), a.size() * 2);
  llmx_copy(gpu, cpu, via_registry.const_data_ptr(), b.data(), b.size() * 2);
  llmx_copy(gpu, cpu, via_helper.const_data_ptr(), c.data(), c.size() * 2);
  EXPECT(std::memcmp(a.data(), b.data(), a.size() * 2) == 0);
  EXPECT(std::memcmp(a.data(), c.data(), a.size() * 2) == 0);
  // Host tensors handed to the direct call are refused, not dereferenced.
  bool threw = false;
  try {
    Tensor hq_t(hq.data(), {S, H, D}, ScalarType::kFP16, cpu);
    llmx_single_mha_attention(direct, hq_t, k, v, std::nullopt, scale);
  } catch (const std::runtime_error &) {
    threw = true;
  }
  EXPECT(threw);
}

// The stream-ordered pool: blocks are zero-filled, tracked by llmx_mem_info
// and reused after a free (the pool's reserved memory does not grow for a
// second request of the same size), and every block is freed the way it was
// allocated, whatever the switch says at the time of the free.
static size_t pool_reserved() {
  cudaMemPool_t pool;
  uint64_t bytes = 0;
  if (cudaDeviceGetDefaultMemPool(&pool, 0) != cudaSuccess) return 0;
  cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &bytes);
  return (size_t)bytes;
}

static bool all_zero_fp16(const Tensor &t) {
  std::vector<uint16_t> h((size_t)t.numel(), 0xFFFF);
  llmx_copy(Device(DeviceType::kCUDA, 0), Device(DeviceType::kCPU), t.const_data_ptr(), h.data(), h.size() * 2);
  for (uint16_t x : h)
    if (x != 0) return false;
  return true;
}

static void pooled_storage() {
  Device gpu(DeviceType::kCUDA, 0), cpu(DeviceType::kCPU);
  EXPECT(!llmx_cuda_pool_enabled());
  Tensor direct({1024}, ScalarType::kFP32, gpu);
  direct.allocate();
  llmx_set_cuda_pool(true);
  EXPECT(llmx_cuda_pool_enabled());
  void *first = nullptr;
  size_t reserved = 0;
  {
    Tensor t({1 << 20}, ScalarType::kFP16, gpu);
    t.allocate();
    first = t.data_ptr();
    EXPECT(llmx_mem_info(first).has_value() && llmx_mem_info(first)->nbytes == (2u << 20));
    EXPECT(all_zero_fp16(t));
    std::vector<uint16_t> ones((size_t)t.numel(), 0x3C00);  // 1.0 in fp16
    llmx_copy(cpu, gpu, ones.data(), t.data_ptr(), ones.size() * 2);
    reserved = pool_reserved();
    EXPECT(reserved >= (2u << 20));
  }
  EXPECT(!llmx_mem_info(first).has_value());
  Tensor again({1 << 20}, ScalarType::kFP16, gpu);
  again.allocate();
  EXPECT(pool_reserved() == reserved);  // served from the freed block
  EXPECT(all_zero_fp16(again));         // re-zeroed, not the previous tensor's ones
  void *d = direct.data_ptr();
  direct = Tensor();  // allocated with cudaMalloc: released with cudaFree
  EXPECT(!llmx_mem_info(d).has_value());
  llmx_set_cuda_pool(false);
  void *a = again.data_ptr();
  again = Tensor();  // allocated from the pool: returned to it
  EXPECT(!llmx_mem_info(a).has_value());
  EXPECT(cudaDeviceSynchronize() == cudaSuccess);
}

int main() {
  tensor_semantics();
  pooled_storage();
  smoke_zero_inputs();
  known_answer_uniform_weights();
  argument_errors_throw();
  registry_conversions();
  registry_attention_matches_direct_call();
  if (g_fail) {
    std::fprintf(stderr, "%d check(s) failed\n", g_fail);
    return 1;
  }
  std::printf("all C++ API checks passed\n");
  return 0;
}
