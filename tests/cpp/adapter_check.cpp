// Exercises include/bfvgpu_ref.hpp, the C++ adapters with the reference's backend-class
// interfaces, compiled with g++ against libbfvgpu.so (tests/test_cpp_adapter.py builds and
// runs it).
//
//   adapter_check host       host-only context: every constructor's validation throws
//                            std::invalid_argument with the library's error name, and a valid
//                            object on a host-only context throws std::runtime_error.
//   adapter_check gpu DIR    device 0: Matrix, Switch, NttBatch and PublicZero on the inputs
//                            in DIR/*.bin, results written to DIR/*_out.bin (the Python test
//                            compares them with the oracle); close() twice; use after close.
// Prints "<mode> ok" and exits 0, or prints the failed check and exits 1.
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <iterator>
#include <stdexcept>
#include <string>
#include <vector>

#include "bfvgpu_ref.hpp"

namespace {

int failures = 0;

void expect(bool ok, const std::string& what) {
  if (!ok) {
    std::cerr << "FAILED: " << what << "\n";
    ++failures;
  }
}

// Runs f, which must throw E with `name` in its message.
template <class E, class F>
void expect_throw(F&& f, const std::string& name, const std::string& what) {
  try {
    f();
  } catch (const E& e) {
    expect(std::string(e.what()).find(name) != std::string::npos, what + ": message '" + e.what() + "'");
    return;
  } catch (const std::exception& e) {
    expect(false, what + ": wrong exception type, '" + e.what() + "'");
    return;
  }
  expect(false, what + ": no exception");
}

std::vector<uint64_t> load(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  std::vector<char> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  std::vector<uint64_t> words(bytes.size() / 8);
  std::memcpy(words.data(), bytes.data(), words.size() * 8);
  return words;
}

void save(const std::string& path, const std::vector<uint64_t>& words) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(words.data()), static_cast<std::streamsize>(words.size() * 8));
}

void host_checks() {
  auto ctx = bfvgpu_ref::Context::art002(-1);
  const size_t n = ctx->n(), dk = ctx->dk(), k = ctx->k();
  std::vector<uint64_t> ct(2 * dk * n, 0);
  // Matrix: shape, canonical residues, then the device requirement
  expect_throw<std::invalid_argument>([&] { matrix_gpu::Matrix m(ctx, std::vector<uint64_t>(7)); },
                                      "MATRIX_GPU_SHAPE", "Matrix rejects a partial ciphertext");
  std::vector<uint64_t> bad = ct;
  bad[5] = ~uint64_t(0);
  expect_throw<std::invalid_argument>([&] { matrix_gpu::Matrix m(ctx, bad); }, "BFVGPU_E_CANONICAL",
                                      "Matrix rejects a residue >= q");
  expect_throw<std::runtime_error>([&] { matrix_gpu::Matrix m(ctx, ct); }, "BFVGPU_E_DEVICE",
                                   "Matrix needs a device context");
  // Switch: element, key shape, device
  std::vector<uint64_t> key(dk * 2 * k * n, 0);
  expect_throw<std::invalid_argument>([&] { prag::experimental_full_switch::Switch s(ctx, key, 4); },
                                      "BFVGPU_E_ELEMENT", "Switch rejects an even element");
  expect_throw<std::invalid_argument>([&] { prag::experimental_full_switch::Switch s(ctx, key, 2 * n + 1); },
                                      "BFVGPU_E_ELEMENT", "Switch rejects an element >= 2n");
  expect_throw<std::invalid_argument>(
      [&] { prag::experimental_full_switch::Switch s(ctx, std::vector<uint64_t>(3), 3); }, "E_SWITCH_SHAPE",
      "Switch rejects a key of the wrong size");
  expect_throw<std::runtime_error>([&] { prag::experimental_full_switch::Switch s(ctx, key, 3); },
                                   "BFVGPU_E_DEVICE", "Switch needs a device context");
  // PublicZero: canonical public key
  std::vector<uint64_t> pk(2 * k * n, 0);
  pk[n] = ~uint64_t(0);
  expect_throw<std::invalid_argument>([&] { prag::enc0_gpu::PublicZero z(ctx, pk); }, "BFVGPU_E_CANONICAL",
                                      "PublicZero rejects a residue >= q");
  // NttBatch: 1..19 batches
  expect_throw<std::invalid_argument>([&] { prag::experimental::ntt::NttBatch b(ctx, false, 20); },
                                      "BFVGPU_E_CONTEXT", "NttBatch rejects 20 batches");
  expect_throw<std::runtime_error>([&] { prag::experimental::ntt::NttBatch b(ctx, true, 1); }, "BFVGPU_E_DEVICE",
                                   "NttBatch needs a device context");
  // TokenWeights: only the ART-002 degree
  std::vector<uint64_t> primes(3);
  const int32_t bits[3] = {36, 36, 37};
  bfvgpu_ref::check(bfvgpu_find_primes(4096, bits, 3, primes.data()));
  auto small = bfvgpu_ref::Context::create(4096, primes, 3, 0, 65537, -1);
  expect_throw<std::invalid_argument>(
      [&] { prag::experimental::resident::TokenWeights t(small, std::vector<uint64_t>(19 * 2 * 3 * 4096)); },
      "BFVGPU_E_CONTEXT", "TokenWeights rejects n = 4096");
  // the context itself validates its parameters
  expect_throw<std::invalid_argument>([&] { bfvgpu_ref::Context::create(1000, primes, 3, 0, 65537, -1); },
                                      "BFVGPU_E_", "Context rejects n = 1000");
}

void gpu_checks(const std::string& dir) {
  auto ctx = bfvgpu_ref::Context::art002(0);
  // Matrix (bfv_matrix.inc:67, :164)
  {
    matrix_gpu::Matrix m(ctx, load(dir + "/cts.bin"));
    const auto ring = load(dir + "/ring.bin");
    save(dir + "/matrix_selective_out.bin", m.evaluate_selective(ring, load(dir + "/targets.bin")));
    save(dir + "/matrix_out.bin", m.evaluate(ring));
    expect(m.device_bytes() > 0, "Matrix device_bytes");
    const auto c = m.close();
    expect(c.closed && c.first_cuda_error == 0 && c.wiped == c.freed && c.wiped > 0, "Matrix close record");
    const auto again = m.close();
    expect(again.closed && again.first_cuda_error == 0, "Matrix close is idempotent");
    expect_throw<std::invalid_argument>([&] { m.evaluate(ring); }, "MATRIX_GPU_SHAPE", "Matrix use after close");
  }
  // Switch::apply
  {
    const auto elt = static_cast<uint32_t>(load(dir + "/elt.bin").at(0));
    prag::experimental_full_switch::Switch s(ctx, load(dir + "/key.bin"), elt);
    save(dir + "/switch_out.bin", s.apply(load(dir + "/ct.bin")));
    expect(s.element() == elt, "Switch element");
    const auto c = s.close();
    expect(c.closed && c.wipe_synchronized_bytes == c.freed_bytes && c.freed_bytes > 0, "Switch close record");
  }
  // NttBatch round trip
  {
    prag::experimental::ntt::NttBatch b(ctx, false, 2);
    const auto in = load(dir + "/ntt_in.bin");
    const auto f = b.transform(in, false);
    save(dir + "/ntt_out.bin", f);
    expect(b.transform(f, true) == in, "NttBatch round trip");
    expect(b.close().closed, "NttBatch close");
  }
  // PublicZero::encrypt_from_samples
  {
    prag::enc0_gpu::PublicZero z(ctx, load(dir + "/pk.bin"));
    prag::enc0_gpu::Samples s;
    s.words = load(dir + "/samples.bin");
    save(dir + "/enc0_out.bin", z.encrypt_from_samples(s));
    expect(z.close().closed, "PublicZero close");
  }
}

}  // namespace

int main(int argc, char** argv) {
  const std::string mode = argc > 1 ? argv[1] : "host";
  try {
    if (mode == "host")
      host_checks();
    else if (mode == "gpu" && argc > 2)
      gpu_checks(argv[2]);
    else {
      std::cerr << "usage: adapter_check host | gpu DIR\n";
      return 2;
    }
  } catch (const std::exception& e) {
    std::cerr << "FAILED: unexpected exception: " << e.what() << "\n";
    return 1;
  }
  if (failures) return 1;
  std::cout << mode << " ok\n";
  return 0;
}
