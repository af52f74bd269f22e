// bfvgpu_ref.hpp -- C++ adapters with the reference's GPU-backend class interfaces.
//
// privacy-rag's protocol engine constructs its GPU backends as C++ classes
// (IV1 = implementation_v1/ of the reference):
//   matrix_gpu::Matrix                          IV1/experiments/matrix_gpu/matrix.hpp:9-24
//   prag::experimental_full_switch::Switch      IV1/experiments/keyswitch_full_gpu/switch.hpp:12-28
//   prag::enc0_gpu::PublicZero                  IV1/native/gpu/enc0/enc0.hpp:15-25
//   prag::experimental::ntt::NttBatch           IV1/native/gpu/client_phase/ntt.hpp:22-40
//   prag::experimental::resident::TokenWeights  IV1/experiments/resident_token_gpu/resident.hpp:23-48
// This header re-creates those classes, with the same names, member functions, argument
// meaning, Cleanup records and exception behaviour, over the C ABI of bfvgpu.h, so a call
// site such as bfv_matrix.inc:67/:164 keeps its shape.  One difference is deliberate: this
// library does not link SEAL, so where a reference constructor takes SEAL objects
// (SEALContext, Ciphertext, GaloisKeys, PublicKey) the adapter takes a bfvgpu_ref::Context
// and the flat little-endian uint64 arrays a SEAL adapter copies out of those objects
// ([I][2][6][n] ciphertexts, [6][2][7][n] keys, [2][7][n] public key).
//
// Errors: a validation failure throws std::invalid_argument, a device, CUDA, state or
// closed-object failure std::runtime_error, each with the library's E_* text (the
// reference throws the same two types).  close() never throws and is idempotent.
// Header-only; link with -lbfvgpu (privacy-rag_b200/lib) and -lcudart.
#ifndef BFVGPU_REF_HPP
#define BFVGPU_REF_HPP

#include <array>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "bfvgpu.h"

namespace bfvgpu_ref {

[[noreturn]] inline void raise(int32_t rc) {
  const char* text = bfvgpu_last_error();
  const std::string msg = std::string(bfvgpu_error_name(rc)) + ": " + (text ? text : "");
  switch (rc) {
    case BFVGPU_E_CUDA:
    case BFVGPU_E_DEVICE:
    case BFVGPU_E_ALLOC:
    case BFVGPU_E_CLOSED:
    case BFVGPU_E_STATE:
      throw std::runtime_error(msg);
    default:
      throw std::invalid_argument(msg);
  }
}
inline void check(int32_t rc) {
  if (rc != BFVGPU_OK) raise(rc);
}

// A parameter context on one device (device = -1: host-only, tables and constants only;
// every object constructor then fails with std::runtime_error after its validation).
// Stands in for the SEALContext the reference's constructors take.
class Context {
 public:
  static std::shared_ptr<Context> art002(int device = 0) {
    bfvgpu_ctx* h = nullptr;
    check(bfvgpu_ctx_create_art002(device, &h));
    return std::shared_ptr<Context>(new Context(h, 16384, 7, 6));
  }
  static std::shared_ptr<Context> create(uint32_t n, const std::vector<uint64_t>& primes, uint32_t data_primes,
                                         uint32_t special_primes, uint64_t plain_modulus, int device = 0) {
    bfvgpu_ctx* h = nullptr;
    check(bfvgpu_ctx_create(n, primes.data(), data_primes, special_primes, plain_modulus, device, &h));
    return std::shared_ptr<Context>(new Context(h, n, data_primes + special_primes, data_primes));
  }
  ~Context() { bfvgpu_ctx_destroy(h_); }
  Context(const Context&) = delete;
  Context& operator=(const Context&) = delete;
  bfvgpu_ctx* get() const { return h_; }
  size_t n() const { return n_; }
  size_t k() const { return k_; }    // primes at the key level
  size_t dk() const { return dk_; }  // data primes
  // Primes below 2^50 on the FP64 pipe (default) or the integer pipe; set before keys are
  // prepared (bfvgpu_ctx_set_fp64).
  void set_fp64(bool on) { check(bfvgpu_ctx_set_fp64(h_, on ? 1 : 0)); }

 private:
  Context(bfvgpu_ctx* h, size_t n, size_t k, size_t dk) : h_(h), n_(n), k_(k), dk_(dk) {}
  bfvgpu_ctx* h_;
  size_t n_, k_, dk_;
};

}  // namespace bfvgpu_ref

// ---- matrix_gpu::Matrix (IV1/experiments/matrix_gpu/matrix.hpp:9-24) ----------------------
namespace matrix_gpu {
constexpr size_t degree = 16384, primes = 6;
struct Cleanup {
  int first_cuda_error = 0;
  size_t wiped = 0, freed = 0;
  bool closed = false;
};
class Matrix {
 public:
  // inputs: [I][2][6][16384] coefficient-form ciphertexts, canonical (matrix.hpp's
  // std::vector<seal::Ciphertext>, flattened); validated, uploaded and transformed once.
  Matrix(std::shared_ptr<bfvgpu_ref::Context> ctx, const std::vector<uint64_t>& inputs) : ctx_(std::move(ctx)) {
    const size_t ct_words = 2 * ctx_->dk() * ctx_->n();
    if (inputs.empty() || inputs.size() % ct_words) throw std::invalid_argument("MATRIX_GPU_SHAPE");
    inputs_ = inputs.size() / ct_words;
    bfvgpu_ref::check(bfvgpu_matrix_open(ctx_->get(), inputs.data(), inputs_, &m_));
  }
  ~Matrix() { bfvgpu_matrix_release(m_); }
  Matrix(const Matrix&) = delete;
  Matrix& operator=(const Matrix&) = delete;
  // Exactly [input_blocks][16384] packed canonical ring-59 coefficients; returns coefficient
  // form [2][6][16384].
  std::vector<uint64_t> evaluate(const std::vector<uint64_t>& ring) {
    check_ring(ring);
    std::vector<uint64_t> out(2 * ctx_->dk() * ctx_->n());
    bfvgpu_ref::check(bfvgpu_matrix_evaluate(m_, ring.data(), out.data()));
    return out;
  }
  // As evaluate, but c0 is zero except at 1..512 strictly increasing targets.
  std::vector<uint64_t> evaluate_selective(const std::vector<uint64_t>& ring, const std::vector<uint64_t>& targets) {
    check_ring(ring);
    std::vector<uint64_t> out(2 * ctx_->dk() * ctx_->n());
    bfvgpu_ref::check(bfvgpu_matrix_evaluate_selective(m_, ring.data(), targets.data(), targets.size(), out.data()));
    return out;
  }
  size_t device_bytes() const {
    uint64_t b = 0;
    return bfvgpu_matrix_device_bytes(m_, &b) == BFVGPU_OK ? static_cast<size_t>(b) : 0;
  }
  Cleanup close() noexcept {
    bfvgpu_cleanup c{};
    bfvgpu_matrix_close(m_, &c);
    return Cleanup{c.first_cuda_error, static_cast<size_t>(c.wiped), static_cast<size_t>(c.freed), c.closed != 0};
  }

 private:
  void check_ring(const std::vector<uint64_t>& ring) const {
    if (ring.size() != inputs_ * ctx_->n()) throw std::invalid_argument("MATRIX_GPU_SHAPE");
  }
  std::shared_ptr<bfvgpu_ref::Context> ctx_;
  bfvgpu_matrix* m_ = nullptr;
  size_t inputs_ = 0;
};
}  // namespace matrix_gpu

// ---- Switch (IV1/experiments/keyswitch_full_gpu/switch.hpp:12-28) ---------------------------
namespace prag::experimental_full_switch {
constexpr size_t degree = 16384;
struct Timing {
  double setup_upload_ms = 0, upload_ms = 0, rns_ntt_ms = 0, product_ms = 0, inverse_ms = 0, moddown_ms = 0,
         download_ms = 0;
  size_t device_bytes = 0, sensitive_bytes = 0;
};
struct Cleanup {
  int first_cuda_error = 0;
  size_t wipe_synchronized_bytes = 0, freed_bytes = 0;
  bool closed = false;
};
class Switch {
 public:
  // key: the GaloisKeys entry of `element`, [6 digits][2][7][n] in NTT form (the words
  // switch.hpp's SEAL constructor copies out); element odd and < 2n.
  Switch(std::shared_ptr<bfvgpu_ref::Context> ctx, const std::vector<uint64_t>& key, uint32_t element)
      : ctx_(std::move(ctx)), element_(element) {
    if (key.size() != ctx_->dk() * 2 * ctx_->k() * ctx_->n()) throw std::invalid_argument("E_SWITCH_SHAPE");
    bfvgpu_ref::check(bfvgpu_switch_open(ctx_->get(), key.data(), element, &s_));
  }
  ~Switch() { bfvgpu_switch_release(s_); }
  Switch(const Switch&) = delete;
  Switch& operator=(const Switch&) = delete;
  // Galois automorphism then keyswitch of one coefficient-form ciphertext [2][6][n] (the
  // automorphism runs on the GPU; the reference permutes on the CPU first).
  std::vector<uint64_t> apply(const std::vector<uint64_t>& ct) {
    check_ct(ct);
    std::vector<uint64_t> out(ct.size());
    bfvgpu_ref::check(bfvgpu_switch_apply(s_, ct.data(), out.data()));
    return out;
  }
  // Acyclic merge of two ciphertexts: this object holds element 1, `difference` element
  // 2^(level+1)+1.
  std::vector<uint64_t> packing_pair(const std::vector<uint64_t>& left, const std::vector<uint64_t>& right,
                                     Switch& difference, unsigned level) {
    check_ct(left);
    check_ct(right);
    std::vector<uint64_t> out(left.size());
    bfvgpu_ref::check(bfvgpu_switch_packing_pair(s_, left.data(), right.data(), difference.s_, level, out.data()));
    return out;
  }
  Timing timing() const {
    Timing t;
    double up = 0, kernel = 0, down = 0;
    if (bfvgpu_switch_timing(s_, &up, &kernel, &down) == BFVGPU_OK) {
      t.upload_ms = up;
      t.product_ms = kernel;  // the fused kernels are not split into the reference's phases
      t.download_ms = down;
    }
    return t;
  }
  Cleanup close() noexcept {
    bfvgpu_cleanup c{};
    bfvgpu_switch_close(s_, &c);
    return Cleanup{c.first_cuda_error, static_cast<size_t>(c.wiped), static_cast<size_t>(c.freed), c.closed != 0};
  }
  uint32_t element() const { return element_; }

 private:
  void check_ct(const std::vector<uint64_t>& ct) const {
    if (ct.size() != 2 * ctx_->dk() * ctx_->n()) throw std::invalid_argument("E_SWITCH_SHAPE");
  }
  std::shared_ptr<bfvgpu_ref::Context> ctx_;
  bfvgpu_switch* s_ = nullptr;
  uint32_t element_;
};
}  // namespace prag::experimental_full_switch

// ---- PublicZero (IV1/native/gpu/enc0/enc0.hpp:15-25) ------------------------------------------
namespace prag::enc0_gpu {
constexpr size_t degree = 16384;
struct Cleanup {
  int first_cuda_error = 0;
  size_t wipe_synchronized_bytes = 0, freed_bytes = 0;
  bool closed = false;
};
// One encryption's ternary u then e0, e1, at the key level, as canonical residues.
struct Samples {
  std::vector<uint64_t> words;
  explicit Samples(size_t words_count = 3 * 7 * degree) : words(words_count) {}
  Samples(const Samples&) = delete;
  Samples& operator=(const Samples&) = delete;
};
class PublicZero {
 public:
  // pk: [2][7][n] NTT form at the key level (the PublicKey's data).
  PublicZero(std::shared_ptr<bfvgpu_ref::Context> ctx, const std::vector<uint64_t>& pk) : ctx_(std::move(ctx)) {
    if (pk.size() != 2 * ctx_->k() * ctx_->n()) throw std::invalid_argument("E_ENC0_SHAPE");
    bfvgpu_ref::check(bfvgpu_enc0_open(ctx_->get(), pk.data(), &e_));
  }
  ~PublicZero() { bfvgpu_enc0_release(e_); }
  PublicZero(const PublicZero&) = delete;
  PublicZero& operator=(const PublicZero&) = delete;
  // Enc(0) = moddown(INTT(NTT(u) . pk_c) + e_c) as [2][6][n] coefficient form.
  std::vector<uint64_t> encrypt_from_samples(const Samples& s) {
    if (s.words.size() != 3 * ctx_->k() * ctx_->n()) throw std::invalid_argument("E_ENC0_SHAPE");
    std::vector<uint64_t> out(2 * ctx_->dk() * ctx_->n());
    bfvgpu_ref::check(bfvgpu_enc0_encrypt_from_samples(e_, s.words.data(), out.data()));
    return out;
  }
  Cleanup close() noexcept {
    bfvgpu_cleanup c{};
    bfvgpu_enc0_close(e_, &c);
    return Cleanup{c.first_cuda_error, static_cast<size_t>(c.wiped), static_cast<size_t>(c.freed), c.closed != 0};
  }

 private:
  std::shared_ptr<bfvgpu_ref::Context> ctx_;
  bfvgpu_enc0* e_ = nullptr;
};
}  // namespace prag::enc0_gpu

// ---- NttBatch (IV1/native/gpu/client_phase/ntt.hpp:22-40) --------------------------------
namespace prag::experimental::ntt {
constexpr size_t degree = 16384;
struct Cleanup {
  int first_cuda_error = 0;
  size_t wipe_synchronized_bytes = 0, freed_bytes = 0;
  bool closed = false;
};
// Canonical-only host API.  Layout [batch][prime][coefficient]; forward: natural -> bit-
// reversed; inverse: bit-reversed -> natural.
class NttBatch {
 public:
  NttBatch(std::shared_ptr<bfvgpu_ref::Context> ctx, bool key_level, size_t batches)
      : ctx_(std::move(ctx)), words_(batches * (key_level ? ctx_->k() : ctx_->dk()) * ctx_->n()) {
    bfvgpu_ref::check(bfvgpu_ntt_open(ctx_->get(), key_level ? 1 : 0, batches, &h_));
    batches_ = batches;
  }
  ~NttBatch() { bfvgpu_ntt_release(h_); }
  NttBatch(const NttBatch&) = delete;
  NttBatch& operator=(const NttBatch&) = delete;
  // Secret key s [6][n] in NTT form (data level); once per object.
  void bind_client_key(const std::vector<uint64_t>& ntt_key) {
    if (ntt_key.size() != ctx_->dk() * ctx_->n()) throw std::invalid_argument("E_CLIENT_KEY_SHAPE");
    bfvgpu_ref::check(bfvgpu_ntt_bind_client_key(h_, ntt_key.data()));
  }
  // c1 [batches][6][n] -> INTT(NTT(c1) . s).
  std::vector<uint64_t> client_phase(const std::vector<uint64_t>& input) {
    if (input.size() != batches_ * ctx_->dk() * ctx_->n()) throw std::invalid_argument("E_NTT_SHAPE");
    std::vector<uint64_t> out(input.size());
    bfvgpu_ref::check(bfvgpu_ntt_client_phase(h_, input.data(), out.data()));
    return out;
  }
  std::vector<uint64_t> transform(const std::vector<uint64_t>& input, bool inverse) {
    if (input.size() != words_) throw std::invalid_argument("E_NTT_SHAPE");
    std::vector<uint64_t> out(words_);
    bfvgpu_ref::check(bfvgpu_ntt_transform(h_, input.data(), out.data(), inverse ? 1 : 0));
    return out;
  }
  Cleanup close() noexcept {
    bfvgpu_cleanup c{};
    bfvgpu_ntt_close(h_, &c);
    return Cleanup{c.first_cuda_error, static_cast<size_t>(c.wiped), static_cast<size_t>(c.freed), c.closed != 0};
  }

 private:
  std::shared_ptr<bfvgpu_ref::Context> ctx_;
  bfvgpu_ntt* h_ = nullptr;
  size_t words_ = 0, batches_ = 0;
};
}  // namespace prag::experimental::ntt

// ---- TokenWeights (IV1/experiments/resident_token_gpu/resident.hpp:23-48) ------------------
namespace prag::experimental::resident {
constexpr size_t degree = 16384, primes = 6, blocks = 19, block_width = 8192;
struct Cleanup {
  int first_cuda_error = 0;
  size_t wipe_synchronized_bytes = 0, freed_bytes = 0;
  bool closed = false;
};
class TokenWeights {
 public:
  // Original coefficient-form ciphertexts [slot <= 4][block = 19][2][6][n]; transformed on
  // the device (the reference transforms them with SEAL on the CPU first).
  TokenWeights(std::shared_ptr<bfvgpu_ref::Context> ctx, const std::vector<uint64_t>& cts) : ctx_(std::move(ctx)) {
    const size_t per_slot = blocks * 2 * ctx_->dk() * ctx_->n();
    if (cts.empty() || cts.size() % per_slot) throw std::invalid_argument("E_GPU_TOKEN_CONTEXT_LAYOUT");
    slots_ = cts.size() / per_slot;
    bfvgpu_ref::check(bfvgpu_token_open(ctx_->get(), cts.data(), slots_, &t_));
  }
  ~TokenWeights() { bfvgpu_token_release(t_); }
  TokenWeights(const TokenWeights&) = delete;
  TokenWeights& operator=(const TokenWeights&) = delete;
  // Exactly [19][8192] canonical ring-59 words with |w| <= 2^20, local shares [slots];
  // returns [slot][2][6][n]: the product, INTT, local share at coefficient 8191, shift
  // (the reference returns it as a device view; here it is downloaded).
  std::vector<uint64_t> evaluate_finished(const std::vector<uint64_t>& weights, const std::vector<uint64_t>& local) {
    if (weights.size() != blocks * block_width || local.size() != slots_)
      throw std::invalid_argument("E_RESIDENT_WEIGHT_SHAPE");
    std::vector<uint64_t> out(slots_ * 2 * ctx_->dk() * ctx_->n());
    bfvgpu_ref::check(bfvgpu_token_evaluate_finished(t_, weights.data(), local.data(), out.data()));
    return out;
  }
  Cleanup close() noexcept {
    bfvgpu_cleanup c{};
    bfvgpu_token_close(t_, &c);
    return Cleanup{c.first_cuda_error, static_cast<size_t>(c.wiped), static_cast<size_t>(c.freed), c.closed != 0};
  }

 private:
  std::shared_ptr<bfvgpu_ref::Context> ctx_;
  bfvgpu_token* t_ = nullptr;
  size_t slots_ = 0;
};
}  // namespace prag::experimental::resident

#endif  // BFVGPU_REF_HPP
