// C ABI of the B200 BFV library: parameter contexts and the reference-shaped objects
// (NttBatch, Matrix, Switch, PublicZero, TokenWeights) over the kernels of kernels.cu.
//
// Object semantics follow the reference backends (IV1 = implementation_v1/):
//   validation before any device work, device state released on any CUDA failure,
//   close() zeroes every sensitive buffer, synchronises, frees it and reports the
//   byte counts (IV1/experiments/matrix_gpu/matrix.cu:72-77, switch.cu:113-127),
//   and there is no CPU fallback.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "bfvgpu.h"
#include "ctx_internal.h"
#include "kernels.cuh"
#include "ntt_core.cuh"

using u128 = unsigned __int128;

namespace bfvgpu {
namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

struct Error {
  int code;
  std::string what;
};
[[noreturn]] void fail(int code, const std::string& what) { throw Error{code, what}; }

void cuda_check(cudaError_t e, const char* where) {
  if (e != cudaSuccess) fail(BFVGPU_E_CUDA, std::string("E_BFVGPU_CUDA: ") + where + ": " + cudaGetErrorString(e));
}

template <class F>
int32_t guard(F&& f) {
  try {
    f();
    return BFVGPU_OK;
  } catch (const Error& e) {
    g_last_error = e.what;
    return e.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "E_HOST_ALLOC";
    return BFVGPU_E_ALLOC;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return BFVGPU_E_ARGUMENT;
  }
}

// ---- host arithmetic for parameter set-up --------------------------------------------
uint64_t mulmod_h(uint64_t a, uint64_t b, uint64_t q) { return (uint64_t)((u128)a * b % q); }
uint64_t powmod_h(uint64_t a, uint64_t e, uint64_t q) {
  uint64_t r = 1 % q;
  a %= q;
  while (e) {
    if (e & 1) r = mulmod_h(r, a, q);
    a = mulmod_h(a, a, q);
    e >>= 1;
  }
  return r;
}
uint64_t shoup_q(uint64_t w, uint64_t q) { return (uint64_t)(((u128)w << 64) / q); }

bool prime_h(uint64_t n) {
  if (n < 2) return false;
  static const uint64_t witnesses[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
  for (uint64_t p : witnesses) {
    if (n % p == 0) return n == p;
  }
  uint64_t d = n - 1;
  int r = 0;
  while ((d & 1) == 0) {
    d >>= 1;
    ++r;
  }
  for (uint64_t a : witnesses) {
    uint64_t x = powmod_h(a, d, n);
    if (x == 1 || x == n - 1) continue;
    bool witness = true;
    for (int i = 1; i < r && witness; ++i) {
      x = mulmod_h(x, x, n);
      if (x == n - 1) witness = false;
    }
    if (witness) return false;
  }
  return true;
}

// Least primitive 2n-th root of unity mod q: among the odd powers of any primitive root.
uint64_t least_root(uint64_t q, uint64_t two_n) {
  uint64_t root = 0;
  for (uint64_t x = 2; x < q && !root; ++x) {
    const uint64_t c = powmod_h(x, (q - 1) / two_n, q);
    if (powmod_h(c, two_n / 2, q) == q - 1) root = c;
  }
  if (!root) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_ROOT");
  const uint64_t sq = mulmod_h(root, root, q);
  uint64_t best = root, cur = root;
  for (uint64_t i = 1; i < two_n / 2; ++i) {
    cur = mulmod_h(cur, sq, q);
    if (cur < best) best = cur;
  }
  return best;
}

uint32_t brv(uint32_t x, int bits) {
  uint32_t r = 0;
  for (int i = 0; i < bits; ++i) r |= ((x >> i) & 1u) << (bits - 1 - i);
  return r;
}

struct DeviceScope {
  int prev = -1;
  bool changed = false;
  explicit DeviceScope(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) {
      cuda_check(cudaSetDevice(dev), "cudaSetDevice");
      changed = true;
    }
  }
  ~DeviceScope() {
    if (changed && prev >= 0) cudaSetDevice(prev);
  }
};

void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

}  // namespace

// ---------------------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------------------
struct Context {
  int device = -1;
  uint32_t n = 0, k = 0, dk = 0;
  int logn = 0;
  uint64_t t = 0;
  std::vector<uint64_t> q;
  std::vector<Modulus> mods;           // integer-pipe records (f64 = 0)
  std::vector<Modulus> mods_f64;       // the same with the FP64 constants of primes < 2^50
  std::vector<uint64_t> fwd_h, inv_h;  // [k][n][2]
  std::vector<double> fwd64_h, inv64_h;  // [k][n][2]
  bool use_f64 = true;                 // primes < 2^50 compute on the FP64 pipe
  const Modulus* dmod_int = nullptr;   // device copies of mods / mods_f64
  const Modulus* dmod_f64 = nullptr;
  uint64_t keys_prepared = 0;          // key preparations issued (fixes the arithmetic mode)
  cudaStream_t stream = nullptr;
  cudaStream_t aux = nullptr;                     // side stream for independent work of one call
  cudaEvent_t fork = nullptr, join = nullptr;     // ordering between a caller's stream and aux
  std::mutex aux_mutex;                           // one call at a time uses aux
  void* dmem = nullptr;  // one public allocation holding all tables
  DevParams P;

  ~Context() {
    if (device >= 0) {
      int prev = -1;
      cudaGetDevice(&prev);
      cudaSetDevice(device);
      if (stream) cudaStreamSynchronize(stream);
      if (aux) cudaStreamSynchronize(aux);
      if (dmem) cudaFree(dmem);
      if (fork) cudaEventDestroy(fork);
      if (join) cudaEventDestroy(join);
      if (aux) cudaStreamDestroy(aux);
      if (stream) cudaStreamDestroy(stream);
      if (prev >= 0) cudaSetDevice(prev);
    }
  }
};

constexpr size_t kErrBytes = 256;

static void build_context(Context& c, uint32_t n, const uint64_t* primes, uint32_t dk, uint32_t special, uint64_t t,
                          int device) {
  if (!primes || n == 0 || (n & (n - 1))) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_DEGREE");
  int logn = 0;
  while ((1u << logn) < n) ++logn;
  if (!logn_supported(logn)) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_DEGREE_UNSUPPORTED");
  if (dk == 0 || dk > 8 || special > 1) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_PRIME_COUNT");
  if (t < 2 || !((t & (t - 1)) == 0 || t < (1ull << 32))) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_PLAIN_MODULUS");
  c.n = n;
  c.logn = logn;
  c.dk = dk;
  c.k = dk + special;
  c.t = t;
  c.q.assign(primes, primes + c.k);
  for (uint32_t i = 0; i < c.k; ++i) {
    const uint64_t qi = c.q[i];
    if (qi >= (1ull << 62) || !prime_h(qi) || (qi - 1) % (2ull * n)) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_PRIME");
    if (qi <= t && i < dk) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_PRIME_BELOW_T");
    for (uint32_t j = 0; j < i; ++j)
      if (c.q[j] == qi) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_PRIME_REPEATED");
  }
  // device check (device == -1: host-only context, tables and constants only)
  if (device != -1) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
      cudaGetLastError();
      fail(BFVGPU_E_DEVICE, "E_BFVGPU_DEVICE_MISSING");
    }
    cudaDeviceProp prop{};
    cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major != 10) fail(BFVGPU_E_DEVICE, "E_BFVGPU_SM100_REQUIRED");
  }

  // ---- tables ----
  c.mods.assign(c.k, Modulus{});
  c.fwd_h.assign((size_t)c.k * n * 2, 0);
  c.inv_h.assign((size_t)c.k * n * 2, 0);
  const uint64_t special_q = special ? c.q[c.k - 1] : 0;
  // Q mod t, then floor(Q/t) mod q_p = -(Q mod t) * t^-1 mod q_p
  uint64_t q_mod_t = 1 % t;
  for (uint32_t i = 0; i < dk; ++i) q_mod_t = (uint64_t)((u128)q_mod_t * (c.q[i] % t) % t);
  for (uint32_t p = 0; p < c.k; ++p) {
    const uint64_t qp = c.q[p];
    Modulus& m = c.mods[p];
    m.q = qp;
    const u128 ratio = (~(u128)0) / qp;
    m.r0 = (uint64_t)ratio;
    m.r1 = (uint64_t)(ratio >> 64);
    const uint64_t ninv = powmod_h(n % qp, qp - 2, qp);
    m.invn = ninv;
    m.invn_q = shoup_q(ninv, qp);
    if (special && p < dk) {
      const uint64_t si = powmod_h(special_q % qp, qp - 2, qp);
      m.inv_special = si;
      m.inv_special_q = shoup_q(si, qp);
      m.half_special_mod = (special_q >> 1) % qp;
    }
    if (p < dk) {
      const uint64_t tinv = powmod_h(t % qp, qp - 2, qp);
      const uint64_t neg_r = (qp - q_mod_t % qp) % qp;
      m.delta = mulmod_h(neg_r, tinv, qp);
      m.delta_q = shoup_q(m.delta, qp);
    }
    const uint64_t psi = least_root(qp, 2ull * n);
    const uint64_t psi_inv = powmod_h(psi, qp - 2, qp);
    uint64_t* f = c.fwd_h.data() + (size_t)p * n * 2;
    uint64_t* r = c.inv_h.data() + (size_t)p * n * 2;
    uint64_t pw = 1;
    for (uint32_t i = 0; i < n; ++i) {
      const uint32_t at = brv(i, logn);
      f[2 * at] = pw;
      f[2 * at + 1] = shoup_q(pw, qp);
      pw = mulmod_h(pw, psi, qp);
    }
    r[0] = 1;
    r[1] = shoup_q(1, qp);
    pw = psi_inv;
    for (uint32_t i = 1; i < n; ++i) {
      const uint32_t at = brv(i - 1, logn) + 1;
      r[2 * at] = pw;
      r[2 * at + 1] = shoup_q(pw, qp);
      pw = mulmod_h(pw, psi_inv, qp);
    }
  }
  // FP64-pipe constants and twiddles (used for the primes below 2^50)
  c.mods_f64 = c.mods;
  c.fwd64_h.assign((size_t)c.k * n * 2, 0.0);
  c.inv64_h.assign((size_t)c.k * n * 2, 0.0);
  for (uint32_t p = 0; p < c.k; ++p) {
    f64_fill_modulus(c.mods_f64[p]);
    if (!c.mods_f64[p].f64) continue;
    const size_t at = (size_t)p * n;
    f64_twiddles(reinterpret_cast<const ulonglong2*>(c.fwd_h.data()) + at, c.q[p], n,
                 reinterpret_cast<double2*>(c.fwd64_h.data()) + at);
    f64_twiddles(reinterpret_cast<const ulonglong2*>(c.inv_h.data()) + at, c.q[p], n,
                 reinterpret_cast<double2*>(c.inv64_h.data()) + at);
  }
  // q_j mod q_p
  std::vector<uint64_t> qjp((size_t)dk * c.k);
  for (uint32_t j = 0; j < dk; ++j)
    for (uint32_t p = 0; p < c.k; ++p) qjp[(size_t)j * c.k + p] = c.q[j] % c.q[p];
  // CRT constants at the data level: Q (dk limbs), Q/q_j (dk limbs), (Q/q_j)^-1 mod q_j
  std::vector<uint64_t> Q(dk + 1, 0), part((size_t)dk * dk, 0), cinv((size_t)dk * 2, 0);
  Q[0] = 1;
  for (uint32_t i = 0; i < dk; ++i) {
    u128 carry = 0;
    for (uint32_t l = 0; l <= dk; ++l) {
      const u128 v = (u128)Q[l] * c.q[i] + carry;
      Q[l] = (uint64_t)v;
      carry = v >> 64;
    }
  }
  for (uint32_t j = 0; j < dk; ++j) {
    u128 rem = 0;
    for (int l = (int)dk; l >= 0; --l) {
      const u128 cur = (rem << 64) | Q[l];
      const uint64_t qd = (uint64_t)(cur / c.q[j]);
      rem = cur % c.q[j];
      if (l < (int)dk) part[(size_t)j * dk + l] = qd;
    }
    uint64_t pm = 1;
    for (uint32_t i = 0; i < dk; ++i)
      if (i != j) pm = mulmod_h(pm, c.q[i] % c.q[j], c.q[j]);
    const uint64_t iv = powmod_h(pm, c.q[j] - 2, c.q[j]);
    cinv[2 * j] = iv;
    cinv[2 * j + 1] = shoup_q(iv, c.q[j]);
  }

  c.P.logn = logn;
  c.P.n = n;
  c.P.k = c.k;
  c.P.dk = dk;
  c.P.t = t;
  c.P.tlog = (t & (t - 1)) == 0 ? __builtin_ctzll(t) : 0;
  c.P.q_mod_t = q_mod_t;
  c.P.upper_half = (t + 1) >> 1;
  if (device == -1) return;

  // ---- upload ----
  c.device = device;
  DeviceScope scope(device);
  cuda_check(configure_kernels(logn), "configure_kernels");
  cuda_check(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking), "cudaStreamCreate");
  cuda_check(cudaStreamCreateWithFlags(&c.aux, cudaStreamNonBlocking), "cudaStreamCreate");
  cuda_check(cudaEventCreateWithFlags(&c.fork, cudaEventDisableTiming), "cudaEventCreate");
  cuda_check(cudaEventCreateWithFlags(&c.join, cudaEventDisableTiming), "cudaEventCreate");
  const size_t mod_bytes = c.k * sizeof(Modulus);
  const size_t tab_bytes = (size_t)c.k * n * 16;
  const size_t qjp_bytes = qjp.size() * 8, part_bytes = part.size() * 8, cinv_bytes = cinv.size() * 8,
               q_bytes = dk * 8;
  auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t total = 2 * up(mod_bytes) + 4 * up(tab_bytes) + up(qjp_bytes) + up(part_bytes) + up(cinv_bytes) +
                       up(q_bytes) + up(kErrBytes);
  cuda_check(cudaMalloc(&c.dmem, total), "cudaMalloc(tables)");
  char* base = (char*)c.dmem;
  size_t off = 0;
  auto place = [&](const void* src, size_t bytes) {
    void* dst = base + off;
    cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c.stream), "upload tables");
    off += up(bytes);
    return dst;
  };
  c.dmod_int = (const Modulus*)place(c.mods.data(), mod_bytes);
  c.dmod_f64 = (const Modulus*)place(c.mods_f64.data(), mod_bytes);
  c.P.mod = c.use_f64 ? c.dmod_f64 : c.dmod_int;
  c.P.fwd = (const ulonglong2*)place(c.fwd_h.data(), tab_bytes);
  c.P.inv = (const ulonglong2*)place(c.inv_h.data(), tab_bytes);
  c.P.fwd64 = (const double2*)place(c.fwd64_h.data(), tab_bytes);
  c.P.inv64 = (const double2*)place(c.inv64_h.data(), tab_bytes);
  c.P.qjp = (const uint64_t*)place(qjp.data(), qjp_bytes);
  c.P.crt_part = (const uint64_t*)place(part.data(), part_bytes);
  c.P.crt_inv = (const uint64_t*)place(cinv.data(), cinv_bytes);
  c.P.crt_q = (const uint64_t*)place(Q.data(), q_bytes);
  static const uint32_t zeros[kErrBytes / 4] = {};
  c.P.err = (uint32_t*)place(zeros, kErrBytes);
  cuda_check(cudaStreamSynchronize(c.stream), "upload tables");
}

// ---------------------------------------------------------------------------------------
// device buffers with wipe accounting
// ---------------------------------------------------------------------------------------
struct Holder {
  Context* ctx = nullptr;
  struct Buf {
    uint64_t* p = nullptr;
    size_t bytes = 0;
  };
  std::vector<Buf> bufs;
  bfvgpu_cleanup cleanup{0, 0, 0, 0};
  bool closing = false;
  uint64_t device_bytes = 0;

  uint64_t* alloc(size_t words) {
    uint64_t* p = nullptr;
    const size_t bytes = words * 8;
    if (cudaMalloc(&p, bytes ? bytes : 8) != cudaSuccess) {
      cudaGetLastError();
      fail(BFVGPU_E_ALLOC, "E_BFVGPU_DEVICE_ALLOC");
    }
    bufs.push_back({p, bytes});
    device_bytes += bytes;
    return p;
  }
  // Replace a buffer by a larger one (old contents wiped first).
  uint64_t* grow(uint64_t* old, size_t words) {
    for (auto& b : bufs)
      if (b.p == old && old) {
        cuda_check(cudaMemsetAsync(b.p, 0, b.bytes, ctx->stream), "wipe");
        cuda_check(cudaStreamSynchronize(ctx->stream), "wipe");
        cleanup.wiped += b.bytes;
        cuda_check(cudaFree(b.p), "cudaFree");
        cleanup.freed += b.bytes;
        device_bytes -= b.bytes;
        b = bufs.back();
        bufs.pop_back();
        break;
      }
    return alloc(words);
  }
  bfvgpu_cleanup release() noexcept {
    closing = true;
    if (cleanup.closed) return cleanup;
    auto ok = [&](cudaError_t e) {
      if (e != cudaSuccess && !cleanup.first_cuda_error) cleanup.first_cuda_error = (int32_t)e;
      return e == cudaSuccess;
    };
    int prev = -1;
    cudaGetDevice(&prev);
    if (!ok(cudaSetDevice(ctx->device))) return cleanup;
    uint64_t queued = 0;
    for (auto& b : bufs)
      if (b.p && ok(cudaMemsetAsync(b.p, 0, b.bytes, ctx->stream))) queued += b.bytes;
    if (ok(cudaStreamSynchronize(ctx->stream))) cleanup.wiped += queued;
    bool all = true;
    for (auto& b : bufs) {
      if (b.p && ok(cudaFree(b.p))) {
        cleanup.freed += b.bytes;
        b.p = nullptr;
      }
      all = all && !b.p;
    }
    cleanup.closed = all ? 1 : 0;
    if (all) bufs.clear();
    if (prev >= 0) cudaSetDevice(prev);
    return cleanup;
  }
  void check_open(const char* what) const {
    if (closing) fail(BFVGPU_E_CLOSED, what);
  }
  // Run f; on any failure release the device state and rethrow (reference: s->release()).
  template <class F>
  void run(F&& f) {
    try {
      f();
    } catch (...) {
      release();
      throw;
    }
  }
  void h2d(uint64_t* dst, const uint64_t* src, size_t words) {
    cuda_check(cudaMemcpyAsync(dst, src, words * 8, cudaMemcpyHostToDevice, ctx->stream), "H2D");
  }
  void d2h(uint64_t* dst, const uint64_t* src, size_t words) {
    cuda_check(cudaMemcpyAsync(dst, src, words * 8, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
  }
  void sync() { cuda_check(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize"); }
};

static void require_device(const Context& c) {
  if (c.device < 0) fail(BFVGPU_E_DEVICE, "E_BFVGPU_HOST_ONLY_CONTEXT");
}

// Every residue of [polys][n] below its prime (poly i: prime offset + i % count), checked
// before any device work.  The scan is branch-free per polynomial (the compiler vectorises
// it) and, for large batches, split over host threads: a config-2 batch of 256 ciphertexts
// is 16.7 M words, which one thread scans in about 15 ms.
static void check_canonical_host(const Context& c, const uint64_t* data, uint64_t polys, uint32_t prime_count,
                                 uint32_t prime_offset) {
  auto scan = [&](uint64_t p0, uint64_t p1) {
    uint64_t bad = 0;
    for (uint64_t i = p0; i < p1; ++i) {
      const uint64_t q = c.q[prime_offset + i % prime_count];
      const uint64_t* a = data + i * c.n;
      uint64_t b = 0;
      for (uint32_t z = 0; z < c.n; ++z) b |= (uint64_t)(a[z] >= q);
      bad |= b;
    }
    return bad != 0;
  };
  constexpr uint64_t kWordsPerThread = uint64_t(1) << 21;  // 16 MiB
  const uint64_t hw = std::max(1u, std::thread::hardware_concurrency());
  const uint64_t threads = std::min<uint64_t>({16, hw, polys, std::max<uint64_t>(1, polys * c.n / kWordsPerThread)});
  bool bad = false;
  if (threads <= 1) {
    bad = scan(0, polys);
  } else {
    std::vector<char> part(threads, 0);
    auto chunk = [&](uint64_t t) { part[t] = scan(polys * t / threads, polys * (t + 1) / threads); };
    std::vector<std::thread> pool;
    uint64_t started = 1;
    try {
      pool.reserve(threads - 1);
      for (; started < threads; ++started) pool.emplace_back(chunk, started);
    } catch (...) {
      // no more threads: this thread scans the chunks that were not handed out
    }
    chunk(0);
    for (uint64_t t = started; t < threads; ++t) chunk(t);
    for (auto& th : pool) th.join();
    bad = std::any_of(part.begin(), part.end(), [](char v) { return v != 0; });
  }
  if (bad) fail(BFVGPU_E_CANONICAL, "E_BFVGPU_CANONICAL_REQUIRED");
}
static void check_ring_host(const uint64_t* ring, uint64_t words) {
  for (uint64_t i = 0; i < words; ++i)
    if (ring[i] >> 59) fail(BFVGPU_E_RING, "MATRIX_GPU_RING");
}
static void wipe_host(uint64_t* p, size_t words) {
  volatile uint64_t* v = p;
  for (size_t i = 0; i < words; ++i) v[i] = 0;
}

}  // namespace bfvgpu

using namespace bfvgpu;

struct bfvgpu_ctx {
  Context c;
};

// ---------------------------------------------------------------------------------------
// NttBatch
// ---------------------------------------------------------------------------------------
struct bfvgpu_ntt {
  Holder h;
  uint32_t primes = 0;
  uint64_t batches = 0, words = 0;
  uint64_t* data = nullptr;
  uint64_t* key = nullptr;
};

// ---------------------------------------------------------------------------------------
// Matrix
// ---------------------------------------------------------------------------------------
struct bfvgpu_matrix {
  Holder h;
  uint64_t inputs = 0;
  uint64_t* input = nullptr;  // [I][2][dk][n] NTT form
  uint64_t* pk = nullptr;     // [2][k][n]
  // per-call buffers sized for `cap` groups
  uint64_t cap = 0;
  uint64_t *ring = nullptr, *weight = nullptr, *out = nullptr, *selected = nullptr, *targets = nullptr,
           *crt = nullptr, *mask = nullptr, *samples = nullptr, *u_ntt = nullptr, *enc0_x = nullptr;
  uint32_t* counts = nullptr;
  uint32_t cap_targets = 0;
};

// ---------------------------------------------------------------------------------------
// Switch
// ---------------------------------------------------------------------------------------
struct bfvgpu_switch {
  Holder h;
  uint32_t elt = 0;
  uint64_t* key = nullptr;
  uint64_t cap = 0;
  uint64_t *in = nullptr, *acc = nullptr, *out = nullptr, *right = nullptr;
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
  double upload_ms = 0, kernel_ms = 0, download_ms = 0;
};

struct bfvgpu_rotations {
  Holder h;
  std::vector<uint32_t> elts;
  uint64_t pw = 0, cap = 0;
  uint64_t* prepared = nullptr;  // [rotations][pw]
  uint64_t *cts = nullptr, *hoisted = nullptr, *x = nullptr, *xs = nullptr, *out[2] = {nullptr, nullptr};
  uint64_t* flag = nullptr;  // canonical-check result of the last upload
  cudaStream_t copy = nullptr;
  cudaEvent_t computed[2] = {nullptr, nullptr}, copied[2] = {nullptr, nullptr};
};

struct bfvgpu_slots {
  Holder h;
  uint32_t baby = 0, giant = 0;
  std::vector<uint32_t> elts;  // baby (3^b), giant (3^(g baby)), swap (2n - 1)
  uint64_t pw = 0;
  uint64_t* prepared = nullptr;  // [baby - 1 + giant - 1 + 1][pw]
  uint64_t* pt = nullptr;        // [giant][baby][dk][n] NTT-form plaintexts
  uint64_t *ct = nullptr, *hoisted = nullptr, *x = nullptr, *rot = nullptr, *in = nullptr, *part = nullptr,
           *giant_out = nullptr, *sum = nullptr, *swapped = nullptr, *out = nullptr;
};

struct bfvgpu_enc0 {
  Holder h;
  uint64_t *pk = nullptr, *samples = nullptr, *u_ntt = nullptr, *x = nullptr, *out = nullptr, *plain = nullptr;
};

struct bfvgpu_token {
  Holder h;
  uint64_t slots = 0;
  uint64_t *input = nullptr, *ring = nullptr, *w = nullptr, *scaled = nullptr, *out = nullptr;
};

extern "C" {

int32_t bfvgpu_version(void) { return 1; }

const char* bfvgpu_error_name(int32_t code) {
  switch (code) {
    case BFVGPU_OK: return "BFVGPU_OK";
    case BFVGPU_E_ARGUMENT: return "BFVGPU_E_ARGUMENT";
    case BFVGPU_E_CONTEXT: return "BFVGPU_E_CONTEXT";
    case BFVGPU_E_SHAPE: return "BFVGPU_E_SHAPE";
    case BFVGPU_E_CANONICAL: return "BFVGPU_E_CANONICAL";
    case BFVGPU_E_RING: return "BFVGPU_E_RING";
    case BFVGPU_E_TARGET_COUNT: return "BFVGPU_E_TARGET_COUNT";
    case BFVGPU_E_TARGET_INDEX: return "BFVGPU_E_TARGET_INDEX";
    case BFVGPU_E_CLOSED: return "BFVGPU_E_CLOSED";
    case BFVGPU_E_CUDA: return "BFVGPU_E_CUDA";
    case BFVGPU_E_DEVICE: return "BFVGPU_E_DEVICE";
    case BFVGPU_E_STATE: return "BFVGPU_E_STATE";
    case BFVGPU_E_BOUND: return "BFVGPU_E_BOUND";
    case BFVGPU_E_ELEMENT: return "BFVGPU_E_ELEMENT";
    case BFVGPU_E_ALLOC: return "BFVGPU_E_ALLOC";
    default: return "BFVGPU_E_UNKNOWN";
  }
}
const char* bfvgpu_last_error(void) { return g_last_error.c_str(); }
uint64_t bfvgpu_launch_count(void) { return g_launches.load(); }

int32_t bfvgpu_find_primes(uint32_t n, const int32_t* bits, uint32_t count, uint64_t* out) {
  return guard([&] {
    if (!bits || !out || !count || count > 16 || !n || (n & (n - 1))) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    for (uint32_t i = 0; i < count; ++i) {
      bool seen = false;
      for (uint32_t j = 0; j < i; ++j) seen |= bits[j] == bits[i];
      if (seen) continue;
      if (bits[i] < 10 || bits[i] > 61) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_PRIME_BITS");
      uint32_t same = 0;
      for (uint32_t j = 0; j < count; ++j) same += bits[j] == bits[i];
      const uint64_t factor = 2ull * n;
      uint64_t v = (((1ull << bits[i]) - 1) / factor) * factor + 1;
      const uint64_t lower = 1ull << (bits[i] - 1);
      std::vector<uint64_t> found;
      while (found.size() < same && v > lower) {
        if (prime_h(v)) found.push_back(v);
        v -= factor;
      }
      if (found.size() != same) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_NOT_ENOUGH_PRIMES");
      size_t take = same;
      for (uint32_t j = 0; j < count; ++j)
        if (bits[j] == bits[i]) out[j] = found[--take];
    }
  });
}

int32_t bfvgpu_ctx_create(uint32_t n, const uint64_t* primes, uint32_t data_primes, uint32_t special_primes,
                          uint64_t plain_modulus, int32_t device, bfvgpu_ctx** out) {
  return guard([&] {
    if (!out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    *out = nullptr;
    auto ctx = std::make_unique<bfvgpu_ctx>();
    build_context(ctx->c, n, primes, data_primes, special_primes, plain_modulus, device);
    *out = ctx.release();
  });
}

int32_t bfvgpu_ctx_create_art002(int32_t device, bfvgpu_ctx** out) {
  static const uint64_t locked[7] = {1152921504599080961ULL, 1152921504600260609ULL, 1152921504604979201ULL,
                                     1152921504605962241ULL, 1152921504606584833ULL, 1152921504606683137ULL,
                                     1152921504606748673ULL};
  return bfvgpu_ctx_create(16384, locked, 6, 1, 1ull << 59, device, out);
}

int32_t bfvgpu_ctx_destroy(bfvgpu_ctx* ctx) {
  delete ctx;
  return BFVGPU_OK;
}

int32_t bfvgpu_ctx_tables(const bfvgpu_ctx* ctx, uint32_t prime, uint64_t* fwd, uint64_t* inv, uint64_t* invn) {
  return guard([&] {
    if (!ctx || prime >= ctx->c.k) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    const auto& c = ctx->c;
    const size_t words = (size_t)c.n * 2;
    if (fwd) std::memcpy(fwd, c.fwd_h.data() + prime * words, words * 8);
    if (inv) std::memcpy(inv, c.inv_h.data() + prime * words, words * 8);
    if (invn) {
      invn[0] = c.mods[prime].invn;
      invn[1] = c.mods[prime].invn_q;
    }
  });
}

int32_t bfvgpu_ctx_moduli(const bfvgpu_ctx* ctx, uint32_t prime, uint64_t* out) {
  return guard([&] {
    if (!ctx || !out || prime >= ctx->c.k) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    std::memcpy(out, ctx->c.use_f64 ? &ctx->c.mods_f64[prime] : &ctx->c.mods[prime], sizeof(Modulus));
  });
}

int32_t bfvgpu_ctx_stream(const bfvgpu_ctx* ctx, void** stream, int32_t* device) {
  return guard([&] {
    if (!ctx) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (stream) *stream = (void*)ctx->c.stream;
    if (device) *device = ctx->c.device;
  });
}

// ---- device-resident -------------------------------------------------------------------
static cudaStream_t pick(const bfvgpu_ctx* ctx, void* s) { return s ? (cudaStream_t)s : ctx->c.stream; }

int32_t bfvgpu_ntt_device(bfvgpu_ctx* ctx, uint64_t* data, uint64_t polys, uint32_t prime_count,
                          uint32_t prime_offset, int32_t inverse, void* stream) {
  return guard([&] {
    if (!ctx || (!data && polys) || !prime_count || prime_offset + prime_count > ctx->c.k)
      fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    cuda_check(launch_ntt(ctx->c.P, data, polys, prime_count, prime_offset, inverse != 0, pick(ctx, stream)),
               "ntt");
    count_launch();
  });
}

uint64_t bfvgpu_keyswitch_scratch_words(const bfvgpu_ctx* ctx, uint64_t count) {
  return ctx ? count * 2 * ctx->c.k * ctx->c.n : 0;
}

int32_t bfvgpu_keyswitch_device(bfvgpu_ctx* ctx, const uint64_t* cts, uint64_t count, const uint64_t* key,
                                uint32_t galois_elt, uint64_t* scratch, uint64_t* out, void* stream) {
  return guard([&] {
    if (!ctx || !cts || !key || !scratch || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    if (!(galois_elt & 1) || galois_elt >= 2 * ctx->c.n) fail(BFVGPU_E_ELEMENT, "E_BFVGPU_GALOIS_ELEMENT");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    cuda_check(launch_keyswitch(ctx->c.P, cts, key, galois_elt, count, scratch, out, pick(ctx, stream)),
               "keyswitch");
    count_launch(2);
  });
}

uint64_t bfvgpu_keyswitch_prepared_words(const bfvgpu_ctx* ctx) {
  return ctx ? ks_prepared_words(ctx->c.k, ctx->c.dk, ctx->c.n) : 0;
}

uint64_t bfvgpu_keyswitch_hoist_words(const bfvgpu_ctx* ctx, uint64_t count) {
  return ctx ? count * ctx->c.dk * ctx->c.k * ctx->c.n + (count + 1) / 2 : 0;
}

int32_t bfvgpu_keyswitch_prepare_device(bfvgpu_ctx* ctx, const uint64_t* keys, const uint32_t* galois_elts,
                                        uint64_t count, uint64_t* prepared, void* stream) {
  return guard([&] {
    if (!ctx || !keys || !galois_elts || !prepared || !count) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    for (uint64_t r = 0; r < count; ++r)
      if (!(galois_elts[r] & 1) || galois_elts[r] >= 2 * ctx->c.n) fail(BFVGPU_E_ELEMENT, "E_BFVGPU_GALOIS_ELEMENT");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    ++ctx->c.keys_prepared;
    cuda_check(launch_ks_keyprep(ctx->c.P, keys, galois_elts, count, prepared, pick(ctx, stream)), "keyprep");
    count_launch(2 * ((count + 255) / 256));
  });
}

int32_t bfvgpu_keyswitch_hoist_device(bfvgpu_ctx* ctx, const uint64_t* cts, uint64_t count, uint64_t* hoisted,
                                      void* stream) {
  return guard([&] {
    if (!ctx || !cts || !hoisted || !count) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    uint32_t* zflag = (uint32_t*)(hoisted + count * ctx->c.dk * ctx->c.k * ctx->c.n);
    cuda_check(launch_ks_hoist(ctx->c.P, cts, count, hoisted, zflag, pick(ctx, stream)), "hoist");
    count_launch();
  });
}

int32_t bfvgpu_keyswitch_rotate_device(bfvgpu_ctx* ctx, const uint64_t* cts, uint64_t count, const uint64_t* hoisted,
                                       const uint64_t* prepared, uint32_t galois_elt, uint64_t* scratch,
                                       uint64_t* out, void* stream) {
  return guard([&] {
    if (!ctx || !cts || !hoisted || !prepared || !scratch || !out || !count)
      fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    if (!(galois_elt & 1) || galois_elt >= 2 * ctx->c.n) fail(BFVGPU_E_ELEMENT, "E_BFVGPU_GALOIS_ELEMENT");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    const uint32_t* zflag = (const uint32_t*)(hoisted + count * ctx->c.dk * ctx->c.k * ctx->c.n);
    cuda_check(launch_ks_rotate(ctx->c.P, cts, count, hoisted, zflag, prepared, galois_elt, scratch, out,
                                pick(ctx, stream)),
               "rotate");
    count_launch(2);
  });
}

uint64_t bfvgpu_keyswitch_rotate_many_scratch_words(const bfvgpu_ctx* ctx, uint64_t count) {
  return ctx ? count * 2ull * ctx->c.k * ctx->c.n + 2 * count * 2ull * ctx->c.n : 0;
}

int32_t bfvgpu_keyswitch_rotate_many_device(bfvgpu_ctx* ctx, const uint64_t* cts, uint64_t count,
                                            const uint64_t* hoisted, const uint64_t* prepared,
                                            const uint32_t* galois_elts, uint64_t elements, uint64_t* scratch,
                                            uint64_t* const* outs, void* stream) {
  return guard([&] {
    if (!ctx || !cts || !hoisted || !prepared || !galois_elts || !scratch || !outs || !count)
      fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    for (uint64_t e = 0; e < elements; ++e) {
      if (!(galois_elts[e] & 1) || galois_elts[e] >= 2 * ctx->c.n) fail(BFVGPU_E_ELEMENT, "E_BFVGPU_GALOIS_ELEMENT");
      if (!outs[e]) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    }
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    const Context& c = ctx->c;
    const uint32_t* zflag = (const uint32_t*)(hoisted + count * c.dk * c.k * c.n);
    uint64_t* xs = scratch + count * 2ull * c.k * c.n;
    cuda_check(launch_ks_rotate_pipe(c.P, cts, count, hoisted, zflag, prepared, galois_elts, elements, scratch, xs,
                                     outs, pick(ctx, stream)),
               "rotate many");
    count_launch(elements ? elements + 1 : 0);
  });
}

int32_t bfvgpu_weights_ntt_device(bfvgpu_ctx* ctx, const uint64_t* ring, uint64_t blocks, uint64_t* out,
                                  void* stream) {
  return guard([&] {
    if (!ctx || !ring || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    cuda_check(launch_lift_ntt(ctx->c.P, ring, out, blocks, pick(ctx, stream)), "lift_ntt");
    count_launch();
  });
}

int32_t bfvgpu_matrix_groups_device(bfvgpu_ctx* ctx, const uint64_t* in, uint64_t inputs, const uint64_t* w,
                                    uint64_t groups, const uint64_t* mask, const uint64_t* enc0_x, uint64_t* out,
                                    void* stream) {
  return guard([&] {
    if (!ctx || !in || !w || !out || !inputs) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (enc0_x && ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    Protect prot{mask, enc0_x};
    cuda_check(launch_mac_intt(ctx->c.P, in, w, out, inputs, groups, prot, pick(ctx, stream)), "mac_intt");
    count_launch();
  });
}

int32_t bfvgpu_ctx_check(bfvgpu_ctx* ctx, uint32_t* flags) {
  return guard([&] {
    if (!ctx || !flags) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    *flags = 0;
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    cuda_check(cudaDeviceSynchronize(), "ctx_check");
    cuda_check(cudaMemcpy(flags, ctx->c.P.err, 4, cudaMemcpyDeviceToHost), "ctx_check");
    cuda_check(cudaMemset(ctx->c.P.err, 0, 4), "ctx_check");
    if (*flags) fail(BFVGPU_E_CUDA, "E_BFVGPU_KERNEL_TIMEOUT");
  });
}

int32_t bfvgpu_ctx_set_reserved_sms(bfvgpu_ctx* ctx, int32_t sms) {
  return guard([&] {
    if (!ctx || sms < 0 || sms > 64) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    ctx->c.P.reserved_sms = sms;
  });
}

int32_t bfvgpu_ctx_set_product_path(bfvgpu_ctx* ctx, int32_t path) {
  return guard([&] {
    if (!ctx || path < 0 || path > 2) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    ctx->c.P.product_path = path;
  });
}

int32_t bfvgpu_ctx_set_fp64(bfvgpu_ctx* ctx, int32_t on) {
  return guard([&] {
    if (!ctx || on < 0 || on > 1) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    Context& c = ctx->c;
    if ((on != 0) != c.use_f64 && c.keys_prepared) fail(BFVGPU_E_STATE, "E_BFVGPU_ARITH_STATE");
    c.use_f64 = on != 0;
    if (c.device >= 0) c.P.mod = c.use_f64 ? c.dmod_f64 : c.dmod_int;
  });
}

int32_t bfvgpu_ctx_set_limb_split(bfvgpu_ctx* ctx, int32_t split) {
  return guard([&] {
    if (!ctx || split < 0 || split > 1) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    ctx->c.P.split_limbs = split;
  });
}

uint64_t bfvgpu_matrix_tiles_scratch_words(const bfvgpu_ctx* ctx, uint64_t tiles, uint64_t groups, int32_t enc0) {
  if (!ctx) return 0;
  // U [items][k][n] + xs [items][2][n] (Enc(0) only) + E [items][2][dk][n]
  const uint64_t items = tiles * groups, n = ctx->c.n;
  return items * ((enc0 ? ctx->c.k + 2 : 0) + 2ull * ctx->c.dk) * n;
}

static void require_product_ring(const Context& c) {
  if (c.n < 32) fail(BFVGPU_E_RING, "E_BFVGPU_PRODUCT_RING");
  for (uint32_t p = 0; p < c.dk; ++p)
    if (c.q[p] >> 60) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_PRODUCT_PRIME");
}

int32_t bfvgpu_matrix_tiles_inputs_device(bfvgpu_ctx* ctx, const uint64_t* cts, uint64_t count, uint64_t* out,
                                          void* stream) {
  return guard([&] {
    if (!ctx || !cts || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    require_product_ring(ctx->c);
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    cuda_check(launch_ntt_split(ctx->c.P, cts, out, count * 2 * ctx->c.dk, pick(ctx, stream)), "ntt_split");
    count_launch();
  });
}

int32_t bfvgpu_matrix_tiles_prepare_pk_device(bfvgpu_ctx* ctx, const uint64_t* pk, uint64_t* pk_prep, void* stream) {
  return guard([&] {
    if (!ctx || !pk || !pk_prep) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    cuda_check(launch_pk_prep(ctx->c.P, pk, reinterpret_cast<ulonglong2*>(pk_prep), pick(ctx, stream)), "pk_prep");
    count_launch();
  });
}

// Scratch of the layer pipeline's output protection for `items` outputs:
// U [items][k][n] and xs [items][2][n] (Enc(0)), then E [items][2][dk][n] (Enc(0) or mask).
struct ProtectScratch {
  uint64_t *U = nullptr, *xs = nullptr, *E = nullptr;
};
static ProtectScratch protect_layout(const Context& c, uint64_t items, bool enc0, bool masked, uint64_t* scratch) {
  ProtectScratch ps;
  if (enc0) {
    ps.U = scratch;
    ps.xs = scratch + items * c.k * (uint64_t)c.n;
  }
  if (enc0 || masked) ps.E = scratch + (enc0 ? items * (c.k + 2) * (uint64_t)c.n : 0);
  return ps;
}
// Enc(0) preparation and the additive output term: they depend only on the key, the
// randomness and the masks, not on the call's inputs.
static void protect_prepare(Context& c, uint64_t items, const uint64_t* masks, const uint64_t* samples,
                            const uint64_t* pk_prep, const ProtectScratch& ps, cudaStream_t st) {
  if (samples) {
    cuda_check(launch_enc0_prep(c.P, samples, reinterpret_cast<const ulonglong2*>(pk_prep), items, ps.U, ps.xs, st),
               "enc0_prep");
    count_launch(2);
  }
  cuda_check(launch_enc0_fin(c.P, samples, ps.xs, masks, items, ps.E, st), "enc0_fin");
  count_launch();
}
// The product and the protected output transform (out doubles as the product accumulator:
// each INTT block reads its whole limb before writing it back).
static void product_finish(Context& c, const uint64_t* in, uint64_t tiles, uint64_t inputs, const uint64_t* w,
                           uint64_t groups, const uint64_t* pk_prep, const ProtectScratch& ps, uint64_t* out,
                           cudaStream_t st, cudaEvent_t before_transform) {
  cuda_check(launch_mac_tiles(c.P, in, tiles, inputs, w, groups, out, st), "mac_tiles");
  count_launch(mac_tiles_launches(tiles));
  if (before_transform) cuda_check(cudaStreamWaitEvent(st, before_transform, 0), "wait");
  cuda_check(launch_intt_protect(c.P, out, tiles * groups, ps.U, reinterpret_cast<const ulonglong2*>(pk_prep), ps.E,
                                 out, st),
             "intt_protect");
  count_launch();
}

static void check_tiles_args(bfvgpu_ctx* ctx, const uint64_t* in, const uint64_t* w, const uint64_t* out,
                             uint64_t inputs, bool enc0, bool masked, const uint64_t* pk_prep,
                             const uint64_t* scratch) {
  if (!ctx || !in || !w || !out || !inputs) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
  require_product_ring(ctx->c);
  if ((enc0 && !pk_prep) || ((enc0 || masked) && !scratch)) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
  if (enc0 && ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
  require_device(ctx->c);
}

int32_t bfvgpu_matrix_tiles_device(bfvgpu_ctx* ctx, const uint64_t* in, uint64_t tiles, uint64_t inputs,
                                   const uint64_t* w, uint64_t groups, const uint64_t* masks, const uint64_t* samples,
                                   const uint64_t* pk_prep, uint64_t* scratch, uint64_t* out, void* stream) {
  return guard([&] {
    check_tiles_args(ctx, in, w, out, inputs, samples != nullptr, masks != nullptr, pk_prep, scratch);
    DeviceScope scope(ctx->c.device);
    Context& c = ctx->c;
    const uint64_t items = tiles * groups;
    const ProtectScratch ps = protect_layout(c, items, samples != nullptr, masks != nullptr, scratch);
    cudaStream_t st = pick(ctx, stream);
    std::lock_guard<std::mutex> lock(c.aux_mutex);
    // the protection runs on the side stream, beside the product, and joins before the
    // output transform
    if (ps.E) {
      cuda_check(cudaEventRecord(c.fork, st), "event");
      cuda_check(cudaStreamWaitEvent(c.aux, c.fork, 0), "wait");
      protect_prepare(c, items, masks, samples, pk_prep, ps, c.aux);
      cuda_check(cudaEventRecord(c.join, c.aux), "event");
    }
    product_finish(c, in, tiles, inputs, w, groups, pk_prep, ps, out, st, ps.E ? c.join : nullptr);
  });
}

int32_t bfvgpu_matrix_tiles_protect_device(bfvgpu_ctx* ctx, uint64_t tiles, uint64_t groups, const uint64_t* masks,
                                           const uint64_t* samples, const uint64_t* pk_prep, uint64_t* scratch,
                                           void* stream) {
  return guard([&] {
    if (!ctx || !scratch || (samples && !pk_prep)) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (samples && ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    require_product_ring(ctx->c);
    require_device(ctx->c);
    if (!samples && !masks) return;
    DeviceScope scope(ctx->c.device);
    Context& c = ctx->c;
    const uint64_t items = tiles * groups;
    protect_prepare(c, items, masks, samples, pk_prep,
                    protect_layout(c, items, samples != nullptr, masks != nullptr, scratch), pick(ctx, stream));
  });
}

int32_t bfvgpu_matrix_tiles_prepared_device(bfvgpu_ctx* ctx, const uint64_t* in, uint64_t tiles, uint64_t inputs,
                                            const uint64_t* w, uint64_t groups, int32_t enc0, int32_t masked,
                                            const uint64_t* pk_prep, const uint64_t* scratch, uint64_t* out,
                                            void* stream) {
  return guard([&] {
    check_tiles_args(ctx, in, w, out, inputs, enc0 != 0, masked != 0, pk_prep, scratch);
    DeviceScope scope(ctx->c.device);
    Context& c = ctx->c;
    const ProtectScratch ps = protect_layout(c, tiles * groups, enc0 != 0, masked != 0, const_cast<uint64_t*>(scratch));
    product_finish(c, in, tiles, inputs, w, groups, pk_prep, ps, out, pick(ctx, stream), nullptr);
  });
}

int32_t bfvgpu_enc0_device(bfvgpu_ctx* ctx, const uint64_t* samples, const uint64_t* pk, uint64_t groups,
                           uint64_t* u_scratch, uint64_t* x_out, void* stream) {
  return guard([&] {
    if (!ctx || !samples || !pk || !u_scratch || !x_out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    cuda_check(launch_enc0_x(ctx->c.P, samples, pk, u_scratch, x_out, groups, pick(ctx, stream)), "enc0");
    count_launch();
  });
}

int32_t bfvgpu_gather_targets_device(bfvgpu_ctx* ctx, const uint64_t* out, uint64_t groups, const uint64_t* targets,
                                     const uint32_t* counts, uint32_t max_count, uint64_t* selected, uint64_t* crt,
                                     void* stream) {
  return guard([&] {
    if (!ctx || !out || !targets || !counts || !selected) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (max_count == 0 || max_count > 512) fail(BFVGPU_E_TARGET_COUNT, "MATRIX_GPU_TARGET_COUNT");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    cuda_check(launch_gather_targets(ctx->c.P, out, targets, counts, max_count, groups, selected, crt, pick(ctx, stream)),
               "gather");
    count_launch();
  });
}

// ---- NttBatch ---------------------------------------------------------------------------
int32_t bfvgpu_ntt_open(bfvgpu_ctx* ctx, int32_t key_level, uint64_t batches, bfvgpu_ntt** out) {
  return guard([&] {
    if (!ctx || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    *out = nullptr;
    if (batches < 1 || batches > 19) fail(BFVGPU_E_CONTEXT, "E_NTT_CONTEXT");
    auto h = std::make_unique<bfvgpu_ntt>();
    h->h.ctx = &ctx->c;
    h->primes = key_level ? ctx->c.k : ctx->c.dk;
    h->batches = batches;
    h->words = batches * h->primes * ctx->c.n;
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    h->h.run([&] { h->data = h->h.alloc(h->words); });
    *out = h.release();
  });
}

int32_t bfvgpu_ntt_transform(bfvgpu_ntt* h, const uint64_t* in, uint64_t* out, int32_t inverse) {
  return guard([&] {
    if (!h || !in || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    h->h.check_open("E_NTT_CLOSED");
    const Context& c = *h->h.ctx;
    check_canonical_host(c, in, h->batches * h->primes, h->primes, 0);
    DeviceScope scope(c.device);
    h->h.run([&] {
      h->h.h2d(h->data, in, h->words);
      cuda_check(launch_ntt(c.P, h->data, h->batches * h->primes, h->primes, 0, inverse != 0, c.stream), "ntt");
      count_launch();
      h->h.d2h(out, h->data, h->words);
      h->h.sync();
    });
  });
}

int32_t bfvgpu_ntt_bind_client_key(bfvgpu_ntt* h, const uint64_t* sk) {
  return guard([&] {
    if (!h || !sk) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    h->h.check_open("E_CLIENT_KEY_STATE");
    if (h->key) fail(BFVGPU_E_STATE, "E_CLIENT_KEY_STATE");
    const Context& c = *h->h.ctx;
    if (h->primes != c.dk) fail(BFVGPU_E_CONTEXT, "E_CLIENT_KEY_CONTEXT");
    check_canonical_host(c, sk, c.dk, c.dk, 0);
    DeviceScope scope(c.device);
    h->h.run([&] {
      h->key = h->h.alloc((size_t)c.dk * c.n);
      h->h.h2d(h->key, sk, (size_t)c.dk * c.n);
      h->h.sync();
    });
  });
}

int32_t bfvgpu_ntt_client_phase(bfvgpu_ntt* h, const uint64_t* in, uint64_t* out) {
  return guard([&] {
    if (!h || !in || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    h->h.check_open("E_CLIENT_KEY_STATE");
    if (!h->key) fail(BFVGPU_E_STATE, "E_CLIENT_KEY_STATE");
    const Context& c = *h->h.ctx;
    check_canonical_host(c, in, h->batches * c.dk, c.dk, 0);
    DeviceScope scope(c.device);
    h->h.run([&] {
      h->h.h2d(h->data, in, h->words);
      cuda_check(launch_client_phase(c.P, h->data, h->key, h->batches, c.stream), "client_phase");
      count_launch();
      h->h.d2h(out, h->data, h->words);
      h->h.sync();
    });
  });
}

int32_t bfvgpu_ntt_close(bfvgpu_ntt* h, bfvgpu_cleanup* cleanup) {
  if (!h) return BFVGPU_E_ARGUMENT;
  const bfvgpu_cleanup c = h->h.release();
  if (cleanup) *cleanup = c;
  return BFVGPU_OK;
}
int32_t bfvgpu_ntt_release(bfvgpu_ntt* h) {
  if (!h) return BFVGPU_OK;
  h->h.release();
  delete h;
  return BFVGPU_OK;
}

// ---- Matrix -----------------------------------------------------------------------------
static void matrix_reserve(bfvgpu_matrix* m, uint64_t groups, uint32_t max_targets) {
  const Context& c = *m->h.ctx;
  const uint64_t n = c.n, dk = c.dk, k = c.k;
  if (groups > m->cap) {
    m->ring = m->h.grow(m->ring, groups * m->inputs * n);
    m->weight = m->h.grow(m->weight, groups * m->inputs * dk * n);
    m->out = m->h.grow(m->out, groups * 2 * dk * n);
    m->mask = m->h.grow(m->mask, groups * n);
    if (k > dk) {
      m->samples = m->h.grow(m->samples, groups * 3 * k * n);
      m->u_ntt = m->h.grow(m->u_ntt, groups * k * n);
      m->enc0_x = m->h.grow(m->enc0_x, groups * 2 * k * n);
    }
    m->cap = groups;
    m->cap_targets = 0;
  }
  if (max_targets > m->cap_targets || !m->targets) {
    const uint32_t mt = max_targets < 512 ? 512 : max_targets;
    m->selected = m->h.grow(m->selected, m->cap * dk * mt);
    m->crt = m->h.grow(m->crt, m->cap * dk * mt);
    m->targets = m->h.grow(m->targets, m->cap * mt);
    m->counts = (uint32_t*)m->h.grow((uint64_t*)m->counts, (m->cap + 1) / 2);
    m->cap_targets = mt;
  }
}

int32_t bfvgpu_matrix_open(bfvgpu_ctx* ctx, const uint64_t* cts, uint64_t inputs, bfvgpu_matrix** out) {
  return guard([&] {
    if (!ctx || !cts || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    *out = nullptr;
    if (inputs < 1 || inputs > 512) fail(BFVGPU_E_CONTEXT, "MATRIX_GPU_CONTEXT");
    const Context& c = ctx->c;
    check_canonical_host(c, cts, inputs * 2 * c.dk, c.dk, 0);
    auto m = std::make_unique<bfvgpu_matrix>();
    m->h.ctx = &ctx->c;
    m->inputs = inputs;
    require_device(c);
    DeviceScope scope(c.device);
    m->h.run([&] {
      const uint64_t words = inputs * 2 * c.dk * c.n;
      m->input = m->h.alloc(words);
      m->h.h2d(m->input, cts, words);
      cuda_check(launch_ntt(c.P, m->input, inputs * 2 * c.dk, c.dk, 0, false, c.stream), "input ntt");
      count_launch();
      matrix_reserve(m.get(), 1, 512);
      m->h.sync();
    });
    *out = m.release();
  });
}

// Runs groups through lift/NTT, MAC/INTT (+ protect), gather.  Host buffers.
static void matrix_run(bfvgpu_matrix* m, uint64_t groups, const uint64_t* ring, const uint64_t* targets,
                       const uint32_t* counts, uint32_t max_count, const uint64_t* mask, const uint64_t* samples,
                       uint64_t* full_out, uint64_t* c1_out, uint64_t* c0_targets, uint64_t* c0_crt) {
  const Context& c = *m->h.ctx;
  const uint64_t n = c.n, dk = c.dk, k = c.k;
  matrix_reserve(m, groups, max_count);
  m->h.h2d(m->ring, ring, groups * m->inputs * n);
  cuda_check(launch_lift_ntt(c.P, m->ring, m->weight, groups * m->inputs, c.stream), "lift_ntt");
  count_launch();
  Protect prot{};
  if (mask) {
    m->h.h2d(m->mask, mask, groups * n);
    prot.mask = m->mask;
  }
  if (samples) {
    m->h.h2d(m->samples, samples, groups * 3 * k * n);
    cuda_check(launch_enc0_x(c.P, m->samples, m->pk, m->u_ntt, m->enc0_x, groups, c.stream), "enc0");
    count_launch();
    prot.enc0_x = m->enc0_x;
  }
  cuda_check(launch_mac_intt(c.P, m->input, m->weight, m->out, m->inputs, groups, prot, c.stream), "mac_intt");
  count_launch();
  if (full_out) {
    m->h.d2h(full_out, m->out, groups * 2 * dk * n);
  }
  if (c1_out) {
    for (uint64_t g = 0; g < groups; ++g) m->h.d2h(c1_out + g * dk * n, m->out + (g * 2 + 1) * dk * n, dk * n);
  }
  if (targets && max_count) {
    // counts is a uint32 array: stage as words
    std::vector<uint64_t> tg(groups * (uint64_t)m->cap_targets, 0);
    for (uint64_t g = 0; g < groups; ++g)
      for (uint32_t i = 0; i < counts[g]; ++i) tg[g * m->cap_targets + i] = targets[g * max_count + i];
    cuda_check(cudaMemcpyAsync(m->targets, tg.data(), tg.size() * 8, cudaMemcpyHostToDevice, c.stream), "H2D");
    cuda_check(cudaMemcpyAsync(m->counts, counts, groups * 4, cudaMemcpyHostToDevice, c.stream), "H2D");
    cuda_check(launch_gather_targets(c.P, m->out, m->targets, m->counts, m->cap_targets, groups, m->selected,
                                     c0_crt ? m->crt : nullptr, c.stream),
               "gather");
    count_launch();
    std::vector<uint64_t> sel(groups * dk * m->cap_targets), crt;
    m->h.d2h(sel.data(), m->selected, sel.size());
    if (c0_crt) {
      crt.resize(groups * (uint64_t)m->cap_targets * dk);
      m->h.d2h(crt.data(), m->crt, crt.size());
    }
    m->h.sync();
    for (uint64_t g = 0; g < groups; ++g) {
      for (uint64_t p = 0; p < dk; ++p)
        for (uint32_t i = 0; i < counts[g]; ++i)
          c0_targets[(g * dk + p) * max_count + i] = sel[(g * dk + p) * m->cap_targets + i];
      if (c0_crt)
        for (uint32_t i = 0; i < counts[g]; ++i)
          for (uint64_t l = 0; l < dk; ++l)
            c0_crt[(g * max_count + i) * dk + l] = crt[(g * m->cap_targets + i) * dk + l];
    }
    wipe_host(sel.data(), sel.size());
  }
  m->h.sync();
}

static void validate_targets(const Context& c, const uint64_t* targets, uint64_t count) {
  if (count == 0 || count > 512) fail(BFVGPU_E_TARGET_COUNT, "MATRIX_GPU_TARGET_COUNT");
  for (uint64_t i = 0; i < count; ++i)
    if (targets[i] >= c.n || (i && targets[i] <= targets[i - 1])) fail(BFVGPU_E_TARGET_INDEX, "MATRIX_GPU_TARGET_INDEX");
}

int32_t bfvgpu_matrix_evaluate(bfvgpu_matrix* m, const uint64_t* ring, uint64_t* out) {
  return guard([&] {
    if (!m || !ring || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (m->h.closing) fail(BFVGPU_E_SHAPE, "MATRIX_GPU_SHAPE");
    const Context& c = *m->h.ctx;
    check_ring_host(ring, m->inputs * c.n);
    DeviceScope scope(c.device);
    m->h.run([&] { matrix_run(m, 1, ring, nullptr, nullptr, 0, nullptr, nullptr, out, nullptr, nullptr, nullptr); });
  });
}

int32_t bfvgpu_matrix_evaluate_selective(bfvgpu_matrix* m, const uint64_t* ring, const uint64_t* targets,
                                         uint64_t count, uint64_t* out) {
  return guard([&] {
    if (!m || !ring || !out || (!targets && count)) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    const Context& c = *m->h.ctx;
    validate_targets(c, targets, count);
    if (m->h.closing) fail(BFVGPU_E_SHAPE, "MATRIX_GPU_SHAPE");
    check_ring_host(ring, m->inputs * c.n);
    const uint64_t n = c.n, dk = c.dk;
    std::vector<uint64_t> c0t(dk * count);
    const uint32_t cnt = (uint32_t)count;
    DeviceScope scope(c.device);
    try {
      m->h.run([&] {
        matrix_run(m, 1, ring, targets, &cnt, cnt, nullptr, nullptr, nullptr, out + dk * n, c0t.data(), nullptr);
      });
    } catch (...) {
      wipe_host(out, 2 * dk * n);
      throw;
    }
    std::memset(out, 0, dk * n * 8);
    for (uint64_t p = 0; p < dk; ++p)
      for (uint64_t i = 0; i < count; ++i) out[p * n + targets[i]] = c0t[p * count + i];
    wipe_host(c0t.data(), c0t.size());
  });
}

int32_t bfvgpu_matrix_bind_public_key(bfvgpu_matrix* m, const uint64_t* pk) {
  return guard([&] {
    if (!m || !pk) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    m->h.check_open("MATRIX_GPU_SHAPE");
    const Context& c = *m->h.ctx;
    if (c.k != c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    if (m->pk) fail(BFVGPU_E_STATE, "E_BFVGPU_KEY_BOUND");
    check_canonical_host(c, pk, 2 * c.k, c.k, 0);
    DeviceScope scope(c.device);
    m->h.run([&] {
      m->pk = m->h.alloc(2 * c.k * c.n);
      m->h.h2d(m->pk, pk, 2 * c.k * c.n);
      m->h.sync();
    });
  });
}

int32_t bfvgpu_matrix_evaluate_groups(bfvgpu_matrix* m, uint64_t groups, const uint64_t* ring,
                                      const uint64_t* targets, const uint32_t* counts, uint32_t max_count,
                                      const uint64_t* mask, const uint64_t* samples, uint64_t* c1_out,
                                      uint64_t* c0_targets, uint64_t* c0_crt) {
  return guard([&] {
    if (!m || !ring || !targets || !counts || !c1_out || !c0_targets || !groups)
      fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    m->h.check_open("MATRIX_GPU_SHAPE");
    const Context& c = *m->h.ctx;
    if (max_count == 0 || max_count > 512) fail(BFVGPU_E_TARGET_COUNT, "MATRIX_GPU_TARGET_COUNT");
    for (uint64_t g = 0; g < groups; ++g) {
      if (counts[g] > max_count) fail(BFVGPU_E_TARGET_COUNT, "MATRIX_GPU_TARGET_COUNT");
      validate_targets(c, targets + g * max_count, counts[g]);
    }
    check_ring_host(ring, groups * m->inputs * c.n);
    if (mask) check_ring_host(mask, groups * c.n);
    if (samples) {
      if (!m->pk) fail(BFVGPU_E_STATE, "E_BFVGPU_PUBLIC_KEY_REQUIRED");
      check_canonical_host(c, samples, groups * 3 * c.k, c.k, 0);
    }
    DeviceScope scope(c.device);
    m->h.run([&] {
      matrix_run(m, groups, ring, targets, counts, max_count, mask, samples, nullptr, c1_out, c0_targets, c0_crt);
    });
  });
}

int32_t bfvgpu_matrix_device_bytes(const bfvgpu_matrix* m, uint64_t* bytes) {
  if (!m || !bytes) return BFVGPU_E_ARGUMENT;
  *bytes = m->h.device_bytes;
  return BFVGPU_OK;
}
int32_t bfvgpu_matrix_close(bfvgpu_matrix* m, bfvgpu_cleanup* cleanup) {
  if (!m) return BFVGPU_E_ARGUMENT;
  const bfvgpu_cleanup c = m->h.release();
  if (cleanup) *cleanup = c;
  return BFVGPU_OK;
}
int32_t bfvgpu_matrix_release(bfvgpu_matrix* m) {
  if (!m) return BFVGPU_OK;
  m->h.release();
  delete m;
  return BFVGPU_OK;
}

// ---- Switch -----------------------------------------------------------------------------
int32_t bfvgpu_switch_open(bfvgpu_ctx* ctx, const uint64_t* key, uint32_t elt, bfvgpu_switch** out) {
  return guard([&] {
    if (!ctx || !key || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    *out = nullptr;
    const Context& c = ctx->c;
    if (c.k != c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_NTT_CONTEXT");
    if (!(elt & 1) || elt >= 2 * c.n) fail(BFVGPU_E_ELEMENT, "E_BFVGPU_GALOIS_ELEMENT");
    check_canonical_host(c, key, (uint64_t)c.dk * 2 * c.k, c.k, 0);
    auto s = std::make_unique<bfvgpu_switch>();
    s->h.ctx = &ctx->c;
    s->elt = elt;
    require_device(c);
    DeviceScope scope(c.device);
    s->h.run([&] {
      const uint64_t words = (uint64_t)c.dk * 2 * c.k * c.n;
      s->key = s->h.alloc(words);
      s->h.h2d(s->key, key, words);
      for (auto& e : s->ev) cuda_check(cudaEventCreate(&e), "cudaEventCreate");
      s->h.sync();
    });
    *out = s.release();
  });
}

// Ciphertexts per launch of Switch::apply_many; bounds an object's working set to
// kSwitchChunk * (2 ct + scratch) words (64 cts at n = 8192, 4+1 primes: 106 MB).
constexpr uint64_t kSwitchChunk = 64;

static void switch_reserve(bfvgpu_switch* s, uint64_t count) {
  if (count > kSwitchChunk) count = kSwitchChunk;
  if (count <= s->cap) return;
  const Context& c = *s->h.ctx;
  const uint64_t ctw = 2ull * c.dk * c.n;
  s->in = s->h.grow(s->in, count * ctw);
  s->out = s->h.grow(s->out, count * ctw);
  s->acc = s->h.grow(s->acc, count * 2 * c.k * c.n);
  s->cap = count;
}

int32_t bfvgpu_switch_apply_many(bfvgpu_switch* s, const uint64_t* cts, uint64_t count, uint64_t* out) {
  return guard([&] {
    if (!s || !cts || !out || !count) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    s->h.check_open("E_SWITCH_CLOSED");
    const Context& c = *s->h.ctx;
    check_canonical_host(c, cts, count * 2 * c.dk, c.dk, 0);
    DeviceScope scope(c.device);
    s->h.run([&] {
      switch_reserve(s, count);
      const uint64_t ctw = 2ull * c.dk * c.n;
      double up = 0, ker = 0, down = 0;
      for (uint64_t first = 0; first < count; first += s->cap) {
        const uint64_t m = count - first < s->cap ? count - first : s->cap;
        cuda_check(cudaEventRecord(s->ev[0], c.stream), "event");
        s->h.h2d(s->in, cts + first * ctw, m * ctw);
        cuda_check(cudaEventRecord(s->ev[1], c.stream), "event");
        cuda_check(launch_keyswitch(c.P, s->in, s->key, s->elt, m, s->acc, s->out, c.stream), "keyswitch");
        count_launch(2);
        cuda_check(cudaEventRecord(s->ev[2], c.stream), "event");
        s->h.d2h(out + first * ctw, s->out, m * ctw);
        cuda_check(cudaEventRecord(s->ev[3], c.stream), "event");
        s->h.sync();
        float a = 0, b = 0, d = 0;
        cudaEventElapsedTime(&a, s->ev[0], s->ev[1]);
        cudaEventElapsedTime(&b, s->ev[1], s->ev[2]);
        cudaEventElapsedTime(&d, s->ev[2], s->ev[3]);
        up += a;
        ker += b;
        down += d;
      }
      s->upload_ms = up;
      s->kernel_ms = ker;
      s->download_ms = down;
    });
  });
}

int32_t bfvgpu_switch_apply(bfvgpu_switch* s, const uint64_t* ct, uint64_t* out) {
  return bfvgpu_switch_apply_many(s, ct, 1, out);
}

int32_t bfvgpu_switch_packing_pair(bfvgpu_switch* s, const uint64_t* left, const uint64_t* right,
                                   bfvgpu_switch* other, uint32_t level, uint64_t* out) {
  return guard([&] {
    if (!s || !other || !left || !right || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    const Context& c = *s->h.ctx;
    if (s == other || s->h.closing || other->h.closing || s->h.ctx != other->h.ctx || (1u << (level + 1)) >= c.n ||
        s->elt != 1 || other->elt != (1u << (level + 1)) + 1)
      fail(BFVGPU_E_STATE, "E_PACK_PAIR_STATE");
    check_canonical_host(c, left, 2 * c.dk, c.dk, 0);
    check_canonical_host(c, right, 2 * c.dk, c.dk, 0);
    DeviceScope scope(c.device);
    try {
      switch_reserve(s, 1);
      switch_reserve(other, 1);
      const uint64_t words = 2ull * c.dk * c.n;
      if (!s->right) s->right = s->h.alloc(words);
      s->h.h2d(s->in, left, words);
      s->h.h2d(s->right, right, words);
      // sum -> s->out (temporarily), diff -> other->in
      cuda_check(launch_packing_prepare(c.P, s->in, s->right, s->out, other->in, level, c.stream), "prepare");
      cuda_check(cudaMemcpyAsync(s->in, s->out, words * 8, cudaMemcpyDeviceToDevice, c.stream), "D2D");
      cuda_check(launch_keyswitch(c.P, s->in, s->key, 1, 1, s->acc, s->out, c.stream), "keyswitch");
      cuda_check(launch_keyswitch(c.P, other->in, other->key, other->elt, 1, other->acc, other->out, c.stream),
                 "keyswitch");
      cuda_check(launch_add(c.P, s->out, other->out, 2 * c.dk, c.stream), "add");
      count_launch(6);
      s->h.d2h(out, s->out, words);
      s->h.sync();
    } catch (...) {
      cudaStreamSynchronize(c.stream);
      s->h.release();
      other->h.release();
      wipe_host(out, 2ull * c.dk * c.n);
      throw;
    }
  });
}

int32_t bfvgpu_switch_timing(const bfvgpu_switch* s, double* upload_ms, double* kernel_ms, double* download_ms) {
  if (!s) return BFVGPU_E_ARGUMENT;
  if (upload_ms) *upload_ms = s->upload_ms;
  if (kernel_ms) *kernel_ms = s->kernel_ms;
  if (download_ms) *download_ms = s->download_ms;
  return BFVGPU_OK;
}
int32_t bfvgpu_switch_close(bfvgpu_switch* s, bfvgpu_cleanup* cleanup) {
  if (!s) return BFVGPU_E_ARGUMENT;
  const bool was_open = !s->h.cleanup.closed;
  const bfvgpu_cleanup c = s->h.release();
  if (was_open && c.closed) {
    for (auto& e : s->ev)
      if (e) {
        cudaEventDestroy(e);
        e = nullptr;
      }
  }
  if (cleanup) *cleanup = c;
  return BFVGPU_OK;
}
int32_t bfvgpu_switch_release(bfvgpu_switch* s) {
  if (!s) return BFVGPU_OK;
  bfvgpu_switch_close(s, nullptr);
  delete s;
  return BFVGPU_OK;
}

// ---- Rotations: one ciphertext batch through many Galois keyswitches -----------------------
// Keys [r][dk][2][k][n] are uploaded and prepared (slot-permuted, with their corrections) once
// at open, as Switch uploads its key at construction; apply uploads the batch once, hoists its
// digit transforms and runs every element, copying each element's results back on a second
// stream while the next element computes (two device output buffers).
int32_t bfvgpu_rotations_open(bfvgpu_ctx* ctx, const uint64_t* keys, const uint32_t* galois_elts, uint64_t count,
                              bfvgpu_rotations** out) {
  return guard([&] {
    if (!ctx || !keys || !galois_elts || !count || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    *out = nullptr;
    const Context& c = ctx->c;
    if (c.k != c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_NTT_CONTEXT");
    for (uint64_t r = 0; r < count; ++r)
      if (!(galois_elts[r] & 1) || galois_elts[r] >= 2 * c.n) fail(BFVGPU_E_ELEMENT, "E_BFVGPU_GALOIS_ELEMENT");
    const uint64_t kw = (uint64_t)c.dk * 2 * c.k * c.n;
    check_canonical_host(c, keys, count * c.dk * 2 * c.k, c.k, 0);
    auto s = std::make_unique<bfvgpu_rotations>();
    s->h.ctx = &ctx->c;
    s->elts.assign(galois_elts, galois_elts + count);
    s->pw = ks_prepared_words(c.k, c.dk, c.n);
    require_device(c);
    DeviceScope scope(c.device);
    s->h.run([&] {
      s->prepared = s->h.alloc(count * s->pw);
      constexpr uint64_t kBatch = 16;
      uint64_t* tmp = s->h.alloc((count < kBatch ? count : kBatch) * kw);
      for (uint64_t first = 0; first < count; first += kBatch) {
        const uint64_t m = count - first < kBatch ? count - first : kBatch;
        s->h.h2d(tmp, keys + first * kw, m * kw);
        ++ctx->c.keys_prepared;
        cuda_check(launch_ks_keyprep(c.P, tmp, s->elts.data() + first, m, s->prepared + first * s->pw, c.stream),
                   "keyprep");
        count_launch(2);
      }
      cuda_check(cudaStreamCreateWithFlags(&s->copy, cudaStreamNonBlocking), "cudaStreamCreate");
      for (int i = 0; i < 2; ++i) {
        cuda_check(cudaEventCreateWithFlags(&s->computed[i], cudaEventDisableTiming), "cudaEventCreate");
        cuda_check(cudaEventCreateWithFlags(&s->copied[i], cudaEventDisableTiming), "cudaEventCreate");
      }
      s->h.sync();
    });
    *out = s.release();
  });
}

int32_t bfvgpu_rotations_apply(bfvgpu_rotations* s, const uint64_t* cts, uint64_t count, uint64_t* out) {
  return guard([&] {
    if (!s || !cts || !out || !count) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    s->h.check_open("E_SWITCH_CLOSED");
    const Context& c = *s->h.ctx;
    DeviceScope scope(c.device);
    // the batch is uploaded, then its residues are checked against their primes on the device
    // (a scan of the batch in HBM instead of the host, ~4 ms for 256 ciphertexts) before any
    // work on it; a rejected batch leaves the object as it was
    const uint64_t ctw = 2ull * c.dk * c.n;
    uint32_t bad = 0;
    s->h.run([&] {
      if (count > s->cap) {
        s->cts = s->h.grow(s->cts, count * ctw);
        s->hoisted = s->h.grow(s->hoisted, count * c.dk * c.k * c.n + (count + 1) / 2);
        s->x = s->h.grow(s->x, count * 2 * c.k * c.n);
        s->xs = s->h.grow(s->xs, 2 * count * 2 * c.n);
        s->out[0] = s->h.grow(s->out[0], count * ctw);
        s->out[1] = s->h.grow(s->out[1], count * ctw);
        s->cap = count;
      }
      if (!s->flag) s->flag = s->h.alloc(1);
      s->h.h2d(s->cts, cts, count * ctw);
      cuda_check(cudaMemsetAsync(s->flag, 0, sizeof(uint32_t), c.stream), "cudaMemsetAsync");
      cuda_check(launch_check_canonical(c.P, s->cts, count * 2 * c.dk, c.dk, 0, reinterpret_cast<uint32_t*>(s->flag),
                                        c.stream),
                 "check");
      count_launch();
      cuda_check(cudaMemcpyAsync(&bad, s->flag, sizeof(uint32_t), cudaMemcpyDeviceToHost, c.stream), "D2H");
      s->h.sync();
    });
    if (bad) fail(BFVGPU_E_CANONICAL, "E_BFVGPU_CANONICAL_REQUIRED");
    s->h.run([&] {
      const uint32_t* zflag = (const uint32_t*)(s->hoisted + count * c.dk * c.k * c.n);
      cuda_check(launch_ks_hoist(c.P, s->cts, count, s->hoisted, (uint32_t*)zflag, c.stream), "hoist");
      count_launch();
      // pipelined rotations: launch r completes element r - 1 into out[(r - 1) & 1], whose
      // previous contents (element r - 3) must have been copied out first; each element's
      // copy-back overlaps the following launches on the copy stream
      const uint64_t m = s->elts.size();
      for (uint64_t r = 0; r <= m; ++r) {
        const int b = (int)((r + 1) & 1);
        if (r >= 3) cuda_check(cudaStreamWaitEvent(c.stream, s->copied[b], 0), "wait");
        cuda_check(launch_ks_rotate_pipe_step(c.P, s->cts, count, s->hoisted, zflag, s->prepared, s->elts.data(), m, r,
                                              s->x, s->xs, s->out[b], c.stream),
                   "rotate");
        count_launch();
        if (r == 0) continue;
        cuda_check(cudaEventRecord(s->computed[b], c.stream), "event");
        cuda_check(cudaStreamWaitEvent(s->copy, s->computed[b], 0), "wait");
        cuda_check(cudaMemcpyAsync(out + (r - 1) * count * ctw, s->out[b], count * ctw * 8, cudaMemcpyDeviceToHost,
                                   s->copy),
                   "D2H");
        cuda_check(cudaEventRecord(s->copied[b], s->copy), "event");
      }
      cuda_check(cudaStreamSynchronize(s->copy), "cudaStreamSynchronize");
      s->h.sync();
    });
  });
}

int32_t bfvgpu_rotations_close(bfvgpu_rotations* s, bfvgpu_cleanup* cleanup) {
  if (!s) return BFVGPU_E_ARGUMENT;
  const bool was_open = !s->h.cleanup.closed;
  if (s->copy) cudaStreamSynchronize(s->copy);
  const bfvgpu_cleanup c = s->h.release();
  if (was_open && c.closed) {
    for (int i = 0; i < 2; ++i) {
      if (s->computed[i]) cudaEventDestroy(s->computed[i]);
      if (s->copied[i]) cudaEventDestroy(s->copied[i]);
      s->computed[i] = s->copied[i] = nullptr;
    }
    if (s->copy) cudaStreamDestroy(s->copy);
    s->copy = nullptr;
  }
  if (cleanup) *cleanup = c;
  return BFVGPU_OK;
}

int32_t bfvgpu_rotations_release(bfvgpu_rotations* s) {
  if (!s) return BFVGPU_OK;
  bfvgpu_rotations_close(s, nullptr);
  delete s;
  return BFVGPU_OK;
}

// ---- slot-packed matrix-vector product (BFV batching, baby-step giant-step diagonals) ---------
// Galois element of a left rotation of both slot rows by r: 3^r mod 2n.
static uint32_t row_rotation_elt(uint64_t r, uint32_t n) {
  const uint64_t m = 2ull * n;
  uint64_t g = 1, b = 3;
  for (r %= n / 2; r; r >>= 1, b = b * b % m)
    if (r & 1) g = g * b % m;
  return (uint32_t)g;
}

int32_t bfvgpu_slots_open(bfvgpu_ctx* ctx, const uint64_t* keys, uint32_t baby, uint32_t giant, const uint64_t* plain,
                          bfvgpu_slots** out) {
  return guard([&] {
    if (!ctx || !keys || !plain || !out || baby < 1 || giant < 1) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    *out = nullptr;
    const Context& c = ctx->c;
    if (c.k != c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_NTT_CONTEXT");
    require_product_ring(c);
    if ((uint64_t)baby * giant > c.n / 2 || baby > 4096 || giant > 4096) fail(BFVGPU_E_SHAPE, "E_SLOTS_SHAPE");
    auto s = std::make_unique<bfvgpu_slots>();
    s->h.ctx = &ctx->c;
    s->baby = baby;
    s->giant = giant;
    for (uint32_t b = 1; b < baby; ++b) s->elts.push_back(row_rotation_elt(b, c.n));
    for (uint32_t g = 1; g < giant; ++g) s->elts.push_back(row_rotation_elt((uint64_t)g * baby, c.n));
    s->elts.push_back(2 * c.n - 1);
    const uint64_t nkeys = s->elts.size(), kw = (uint64_t)c.dk * 2 * c.k * c.n;
    check_canonical_host(c, keys, nkeys * c.dk * 2 * c.k, c.k, 0);
    s->pw = ks_prepared_words(c.k, c.dk, c.n);
    require_device(c);
    DeviceScope scope(c.device);
    s->h.run([&] {
      const uint64_t ctw = 2ull * c.dk * c.n, most = baby > giant ? baby : giant;
      s->prepared = s->h.alloc(nkeys * s->pw);
      constexpr uint64_t kBatch = 16;
      uint64_t* tmp = s->h.alloc((nkeys < kBatch ? nkeys : kBatch) * kw);
      for (uint64_t first = 0; first < nkeys; first += kBatch) {
        const uint64_t m = nkeys - first < kBatch ? nkeys - first : kBatch;
        s->h.h2d(tmp, keys + first * kw, m * kw);
        ++ctx->c.keys_prepared;
        cuda_check(launch_ks_keyprep(c.P, tmp, s->elts.data() + first, m, s->prepared + first * s->pw, c.stream),
                   "keyprep");
        count_launch(2);
      }
      s->pt = s->h.alloc((uint64_t)giant * baby * c.dk * c.n);
      cuda_check(launch_lift_ntt(c.P, plain, s->pt, (uint64_t)giant * baby, c.stream), "lift_ntt");
      count_launch();
      s->ct = s->h.alloc(ctw);
      s->hoisted = s->h.alloc(most * c.dk * c.k * c.n + (most + 1) / 2);
      s->x = s->h.alloc(most * 2 * c.k * c.n);
      s->rot = s->h.alloc(baby * ctw);
      s->in = s->h.alloc(baby * ctw);
      s->part = s->h.alloc(giant * ctw);
      s->giant_out = s->h.alloc(giant * ctw);
      s->sum = s->h.alloc(ctw);
      s->swapped = s->h.alloc(ctw);
      s->out = s->h.alloc(ctw);
      s->h.sync();
    });
    *out = s.release();
  });
}

// One product on the context's device: ct [2][dk][n] -> out [2][dk][n] (device pointers).
static void slots_eval(bfvgpu_slots* s, const uint64_t* ct, uint64_t* out, cudaStream_t st) {
  const Context& c = *s->h.ctx;
  const uint64_t ctw = 2ull * c.dk * c.n, B = s->baby, G = s->giant;
  uint32_t* zflag = (uint32_t*)(s->hoisted + (B > G ? B : G) * c.dk * c.k * c.n);
  // baby steps: rot[b] = rotate(ct, b) from one hoisted decomposition
  cuda_check(cudaMemcpyAsync(s->rot, ct, ctw * 8, cudaMemcpyDeviceToDevice, st), "D2D");
  if (B > 1) {
    cuda_check(launch_ks_hoist(c.P, ct, 1, s->hoisted, zflag, st), "hoist");
    cuda_check(launch_ks_rotate_multi(c.P, ct, 1, s->hoisted, zflag, s->prepared, s->elts.data(), B - 1, 0, s->x,
                                      s->rot + ctw, st),
               "rotate");
    count_launch(1 + 2 * ((B - 1 + 255) / 256));
  }
  // part[g] = sum_b pt[g][b] . rot[b] (coefficient form)
  cuda_check(launch_ntt_split(c.P, s->rot, s->in, B * 2 * c.dk, st), "ntt_split");
  cuda_check(launch_mac_tiles(c.P, s->in, 1, B, s->pt, G, s->part, st), "mac_tiles");
  cuda_check(launch_intt_protect(c.P, s->part, G, nullptr, nullptr, nullptr, s->part, st), "intt_protect");
  count_launch(2 + mac_tiles_launches(1));
  // giant steps: giant_out[g] = rotate(part[g], g * baby), paired from one hoist of parts 1..G-1
  cuda_check(cudaMemcpyAsync(s->giant_out, s->part, ctw * 8, cudaMemcpyDeviceToDevice, st), "D2D");
  if (G > 1) {
    cuda_check(launch_ks_hoist(c.P, s->part + ctw, G - 1, s->hoisted, zflag, st), "hoist");
    cuda_check(launch_ks_rotate_multi(c.P, s->part + ctw, G - 1, s->hoisted, zflag, s->prepared + (B - 1) * s->pw,
                                      s->elts.data() + (B - 1), G - 1, 1, s->x, s->giant_out + ctw, st),
               "rotate");
    count_launch(1 + 2 * ((G - 1 + 255) / 256));
  }
  cuda_check(launch_sum_cts(c.P, s->giant_out, G, s->sum, st), "sum");
  // row swap: out = sum + sigma_{2n-1}(sum)
  cuda_check(launch_ks_hoist(c.P, s->sum, 1, s->hoisted, zflag, st), "hoist");
  cuda_check(launch_ks_rotate_multi(c.P, s->sum, 1, s->hoisted, zflag, s->prepared + (B + G - 2) * s->pw,
                                    s->elts.data() + (B + G - 2), 1, 1, s->x, s->swapped, st),
             "rotate");
  cuda_check(cudaMemcpyAsync(out, s->sum, ctw * 8, cudaMemcpyDeviceToDevice, st), "D2D");
  cuda_check(launch_add(c.P, out, s->swapped, 2 * c.dk, st), "add");
  count_launch(5);
}

int32_t bfvgpu_slots_apply_device(bfvgpu_slots* s, const uint64_t* ct, uint64_t* out, void* stream) {
  return guard([&] {
    if (!s || !ct || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    s->h.check_open("E_SWITCH_CLOSED");
    DeviceScope scope(s->h.ctx->device);
    s->h.run([&] { slots_eval(s, ct, out, stream ? (cudaStream_t)stream : s->h.ctx->stream); });
  });
}

int32_t bfvgpu_slots_apply(bfvgpu_slots* s, const uint64_t* ct, uint64_t* out) {
  return guard([&] {
    if (!s || !ct || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    s->h.check_open("E_SWITCH_CLOSED");
    const Context& c = *s->h.ctx;
    check_canonical_host(c, ct, 2 * c.dk, c.dk, 0);
    DeviceScope scope(c.device);
    s->h.run([&] {
      const uint64_t ctw = 2ull * c.dk * c.n;
      s->h.h2d(s->ct, ct, ctw);
      slots_eval(s, s->ct, s->out, c.stream);
      s->h.d2h(out, s->out, ctw);
      s->h.sync();
    });
  });
}

int32_t bfvgpu_slots_close(bfvgpu_slots* s, bfvgpu_cleanup* cleanup) {
  if (!s) return BFVGPU_E_ARGUMENT;
  const bfvgpu_cleanup c = s->h.release();
  if (cleanup) *cleanup = c;
  return BFVGPU_OK;
}

int32_t bfvgpu_slots_release(bfvgpu_slots* s) {
  if (!s) return BFVGPU_OK;
  bfvgpu_slots_close(s, nullptr);
  delete s;
  return BFVGPU_OK;
}

// ---- PublicZero -------------------------------------------------------------------------
int32_t bfvgpu_enc0_open(bfvgpu_ctx* ctx, const uint64_t* pk, bfvgpu_enc0** out) {
  return guard([&] {
    if (!ctx || !pk || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    *out = nullptr;
    const Context& c = ctx->c;
    if (c.k != c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_NTT_CONTEXT");
    check_canonical_host(c, pk, 2 * c.k, c.k, 0);
    auto e = std::make_unique<bfvgpu_enc0>();
    e->h.ctx = &ctx->c;
    require_device(c);
    DeviceScope scope(c.device);
    e->h.run([&] {
      const uint64_t n = c.n, k = c.k, dk = c.dk;
      e->pk = e->h.alloc(2 * k * n);
      e->samples = e->h.alloc(3 * k * n);
      e->u_ntt = e->h.alloc(k * n);
      e->x = e->h.alloc(2 * k * n);
      e->out = e->h.alloc(2 * dk * n);
      e->h.h2d(e->pk, pk, 2 * k * n);
      e->h.sync();
    });
    *out = e.release();
  });
}

int32_t bfvgpu_enc0_encrypt_from_samples(bfvgpu_enc0* e, const uint64_t* samples, uint64_t* out) {
  return guard([&] {
    if (!e || !samples || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    e->h.check_open("E_SWITCH_CLOSED");
    const Context& c = *e->h.ctx;
    check_canonical_host(c, samples, 3 * c.k, c.k, 0);
    DeviceScope scope(c.device);
    e->h.run([&] {
      const uint64_t n = c.n, k = c.k, dk = c.dk;
      e->h.h2d(e->samples, samples, 3 * k * n);
      cuda_check(launch_enc0_x(c.P, e->samples, e->pk, e->u_ntt, e->x, 1, c.stream), "enc0");
      cuda_check(launch_moddown(c.P, e->x, e->out, 1, c.stream), "moddown");
      count_launch(2);
      e->h.d2h(out, e->out, 2 * dk * n);
      // per-call sensitive scratch is wiped after use (enc0.cu:138)
      cuda_check(cudaMemsetAsync(e->samples, 0, 3 * k * n * 8, c.stream), "wipe");
      cuda_check(cudaMemsetAsync(e->u_ntt, 0, k * n * 8, c.stream), "wipe");
      cuda_check(cudaMemsetAsync(e->x, 0, 2 * k * n * 8, c.stream), "wipe");
      cuda_check(cudaMemsetAsync(e->out, 0, 2 * dk * n * 8, c.stream), "wipe");
      e->h.sync();
    });
  });
}
int32_t bfvgpu_enc0_encrypt_plain(bfvgpu_enc0* e, const uint64_t* samples, const uint64_t* plain, uint64_t count,
                                  uint64_t* out) {
  return guard([&] {
    if (!e || !samples || !out || (!plain && count)) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    e->h.check_open("E_SWITCH_CLOSED");
    const Context& c = *e->h.ctx;
    if (count == 0 || count > c.n) fail(BFVGPU_E_SHAPE, "E_BFV_PACKED_SHAPE");
    for (uint64_t i = 0; i < count; ++i)
      if (plain[i] >= c.t) fail(BFVGPU_E_RING, "E_BFV_INPUT_PLAIN");
    check_canonical_host(c, samples, 3 * c.k, c.k, 0);
    DeviceScope scope(c.device);
    e->h.run([&] {
      const uint64_t n = c.n, k = c.k, dk = c.dk;
      if (!e->plain) e->plain = e->h.alloc(n);
      e->h.h2d(e->samples, samples, 3 * k * n);
      e->h.h2d(e->plain, plain, count);
      cuda_check(launch_enc0_x(c.P, e->samples, e->pk, e->u_ntt, e->x, 1, c.stream), "enc0");
      cuda_check(launch_moddown(c.P, e->x, e->out, 1, c.stream), "moddown");
      cuda_check(launch_add_plain(c.P, e->out, e->plain, count, c.stream), "add_plain");
      count_launch(3);
      e->h.d2h(out, e->out, 2 * dk * n);
      cuda_check(cudaMemsetAsync(e->samples, 0, 3 * k * n * 8, c.stream), "wipe");
      cuda_check(cudaMemsetAsync(e->u_ntt, 0, k * n * 8, c.stream), "wipe");
      cuda_check(cudaMemsetAsync(e->x, 0, 2 * k * n * 8, c.stream), "wipe");
      cuda_check(cudaMemsetAsync(e->out, 0, 2 * dk * n * 8, c.stream), "wipe");
      cuda_check(cudaMemsetAsync(e->plain, 0, n * 8, c.stream), "wipe");
      e->h.sync();
    });
  });
}

uint64_t bfvgpu_encrypt_many_scratch_words(const bfvgpu_ctx* ctx, uint64_t cts) {
  return ctx ? cts * 3ull * ctx->c.k * ctx->c.n : 0;
}

int32_t bfvgpu_encrypt_many_device(bfvgpu_ctx* ctx, const uint64_t* samples, const uint64_t* pk, const uint64_t* plain,
                                   uint64_t cts, uint64_t* scratch, uint64_t* out, void* stream) {
  return guard([&] {
    if (!ctx || !samples || !pk || !plain || !scratch || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    if (cts * ctx->c.k > 0x7fffffffull) fail(BFVGPU_E_SHAPE, "E_BFV_PACKED_SHAPE");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    uint64_t* u_ntt = scratch;
    uint64_t* x = scratch + cts * (uint64_t)ctx->c.k * ctx->c.n;
    cuda_check(launch_encrypt_many(ctx->c.P, samples, pk, plain, cts, u_ntt, x, out, pick(ctx, stream)),
               "encrypt_many");
    count_launch(3);
  });
}

uint64_t bfvgpu_protect_scratch_words(const bfvgpu_ctx* ctx, uint64_t count) {
  return ctx ? count * 3ull * ctx->c.k * ctx->c.n : 0;
}

int32_t bfvgpu_protect_device(bfvgpu_ctx* ctx, const uint64_t* cts, uint64_t count, const uint64_t* masks,
                              const uint64_t* samples, const uint64_t* pk, uint64_t* scratch, uint64_t* out,
                              void* stream) {
  return guard([&] {
    if (!ctx || !cts || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (samples && (!pk || !scratch)) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (samples && ctx->c.k != ctx->c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    if (count * ctx->c.k > 0x7fffffffull) fail(BFVGPU_E_SHAPE, "E_BFV_PACKED_SHAPE");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    uint64_t* u_ntt = scratch;
    uint64_t* x = scratch ? scratch + count * (uint64_t)ctx->c.k * ctx->c.n : nullptr;
    cuda_check(launch_protect_ct(ctx->c.P, cts, count, masks, samples, pk, u_ntt, x, out, pick(ctx, stream)),
               "protect");
    count_launch(samples ? 2 : 1);
  });
}

uint64_t bfvgpu_token_finish_scratch_words(const bfvgpu_ctx* ctx, uint64_t slots) {
  if (!ctx) return 0;
  return slots * (3ull * ctx->c.k * ctx->c.n + 512 + 512ull * ctx->c.dk) + (slots + 1) / 2;
}

int32_t bfvgpu_token_finish_device(bfvgpu_ctx* ctx, const uint64_t* packed, uint64_t slots, const uint64_t* masks,
                                   const uint64_t* samples, const uint64_t* pk, uint64_t* scratch, uint64_t* out,
                                   uint64_t* c0_crt, void* stream) {
  return guard([&] {
    if (!ctx || !packed || !masks || !samples || !pk || !scratch || !out || !c0_crt)
      fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    const Context& c = ctx->c;
    if (c.n != 16384 || c.k != c.dk + 1 || c.dk > 8) fail(BFVGPU_E_CONTEXT, "E_TOKEN_CONTEXT");
    if (slots < 1 || slots > 4) fail(BFVGPU_E_SHAPE, "E_TOKEN_BATCH_SHAPE");
    require_device(c);
    DeviceScope scope(c.device);
    const cudaStream_t st = pick(ctx, stream);
    uint64_t* u_ntt = scratch;
    uint64_t* x = u_ntt + slots * (uint64_t)c.k * c.n;
    uint64_t* targets = x + slots * 2ull * c.k * c.n;
    uint64_t* selected = targets + slots * 512;
    uint32_t* counts = reinterpret_cast<uint32_t*>(selected + slots * 512ull * c.dk);
    cuda_check(launch_protect_ct(c.P, packed, slots, masks, samples, pk, u_ntt, x, out, st), "token finish protect");
    cuda_check(launch_packed_targets(targets, counts, slots, st), "token finish targets");
    cuda_check(launch_gather_targets(c.P, out, targets, counts, 512, slots, selected, c0_crt, st), "token finish CRT");
    count_launch(4);
  });
}

int32_t bfvgpu_enc0_close(bfvgpu_enc0* e, bfvgpu_cleanup* cleanup) {
  if (!e) return BFVGPU_E_ARGUMENT;
  const bfvgpu_cleanup c = e->h.release();
  if (cleanup) *cleanup = c;
  return BFVGPU_OK;
}
int32_t bfvgpu_enc0_release(bfvgpu_enc0* e) {
  if (!e) return BFVGPU_OK;
  e->h.release();
  delete e;
  return BFVGPU_OK;
}

// ---- TokenWeights -----------------------------------------------------------------------
int32_t bfvgpu_token_open(bfvgpu_ctx* ctx, const uint64_t* cts, uint64_t slots, bfvgpu_token** out) {
  return guard([&] {
    if (!ctx || !cts || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    *out = nullptr;
    const Context& c = ctx->c;
    if (c.logn != 14 || slots < 1 || slots > 4) fail(BFVGPU_E_CONTEXT, "E_GPU_TOKEN_CONTEXT_LAYOUT");
    constexpr uint64_t blocks = 19;
    check_canonical_host(c, cts, slots * blocks * 2 * c.dk, c.dk, 0);
    auto t = std::make_unique<bfvgpu_token>();
    t->h.ctx = &ctx->c;
    t->slots = slots;
    require_device(c);
    DeviceScope scope(c.device);
    t->h.run([&] {
      const uint64_t n = c.n, dk = c.dk, ctw = 2 * dk * n;
      t->input = t->h.alloc(blocks * slots * ctw);
      // reference layout is [block][slot][2][dk][n]; the caller's is [slot][block][...]
      for (uint64_t s = 0; s < slots; ++s)
        for (uint64_t b = 0; b < blocks; ++b)
          t->h.h2d(t->input + (b * slots + s) * ctw, cts + (s * blocks + b) * ctw, ctw);
      cuda_check(launch_ntt(c.P, t->input, blocks * slots * 2 * dk, dk, 0, false, c.stream), "input ntt");
      count_launch();
      t->ring = t->h.alloc(blocks * 8192);
      t->w = t->h.alloc(blocks * dk * n);
      t->scaled = t->h.alloc(slots * dk);
      t->out = t->h.alloc(slots * ctw);
      t->h.sync();
    });
    *out = t.release();
  });
}

int32_t bfvgpu_token_evaluate_finished(bfvgpu_token* t, const uint64_t* ring, const uint64_t* local, uint64_t* out) {
  return guard([&] {
    if (!t || !ring || !local || !out) fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    t->h.check_open("E_RESIDENT_CLOSED");
    const Context& c = *t->h.ctx;
    constexpr uint64_t modulus = 1ull << 59, bound = 1ull << 20;
    for (uint64_t i = 0; i < 19ull * 8192; ++i)
      if (ring[i] >= modulus || (ring[i] > bound && ring[i] < modulus - bound))
        fail(BFVGPU_E_BOUND, "E_RESIDENT_WEIGHT_BOUND");
    // Delta-scaled local shares (resident/seal_adapter.cpp:43-52), host side
    std::vector<uint64_t> scaled(t->slots * c.dk);
    for (uint64_t s = 0; s < t->slots; ++s) {
      const uint64_t m = local[s];
      if (m >= modulus) fail(BFVGPU_E_RING, "E_GPU_TOKEN_CONTEXT_LAYOUT");
      for (uint64_t p = 0; p < c.dk; ++p)
        scaled[s * c.dk + p] = scale_plain_coeff(m, c.P.q_mod_t, c.P.upper_half, c.t, c.P.tlog, c.mods[p]);
    }
    DeviceScope scope(c.device);
    t->h.run([&] {
      t->h.h2d(t->ring, ring, 19 * 8192);
      t->h.h2d(t->scaled, scaled.data(), scaled.size());
      cuda_check(launch_token_evaluate(c.P, t->input, t->slots, t->ring, t->scaled, t->w, nullptr, t->out, c.stream),
                 "token");
      count_launch(2);
      t->h.d2h(out, t->out, t->slots * 2 * c.dk * c.n);
      t->h.sync();
    });
    wipe_host(scaled.data(), scaled.size());
  });
}
uint64_t bfvgpu_token_many_scratch_words(const bfvgpu_ctx* ctx, uint64_t coords, uint64_t slots) {
  return ctx ? coords * (19ull * ctx->c.dk * ctx->c.n + slots * ctx->c.dk) : 0;
}

int32_t bfvgpu_token_evaluate_many_device(bfvgpu_ctx* ctx, const uint64_t* inputs, uint64_t slots,
                                          const uint64_t* ring, uint64_t coords, const uint64_t* local,
                                          uint64_t* scratch, uint64_t* out, void* stream) {
  return guard([&] {
    if (!ctx || !inputs || !ring || !local || !scratch || !out || !slots || slots > 4)
      fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    if (ctx->c.n != 16384) fail(BFVGPU_E_CONTEXT, "E_GPU_TOKEN_CONTEXT_LAYOUT");
    require_device(ctx->c);
    DeviceScope scope(ctx->c.device);
    uint64_t* w = scratch;
    uint64_t* scaled = scratch + coords * 19ull * ctx->c.dk * ctx->c.n;
    cuda_check(launch_token_evaluate_many(ctx->c.P, inputs, slots, ring, coords, local, scaled, w, out,
                                          pick(ctx, stream)),
               "token_many");
    count_launch(3);
  });
}

uint64_t bfvgpu_packing_level_scratch_words(const bfvgpu_ctx* ctx, uint64_t count) {
  return ctx ? count * (6ull * ctx->c.dk * ctx->c.n + 2ull * ctx->c.k * ctx->c.n) : 0;
}

int32_t bfvgpu_packing_level_device(bfvgpu_ctx* ctx, const uint64_t* in, uint64_t pairs, uint64_t slots,
                                    uint32_t level, const uint64_t* key_one, const uint64_t* key_level,
                                    uint64_t* scratch, uint64_t* out, void* stream) {
  return guard([&] {
    if (!ctx || !in || !key_one || !key_level || !scratch || !out || !pairs || !slots)
      fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
    const Context& c = ctx->c;
    if (c.k != c.dk + 1) fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
    if ((2ull << level) >= c.n) fail(BFVGPU_E_STATE, "E_PACK_PAIR_STATE");
    require_device(c);
    DeviceScope scope(c.device);
    const uint64_t count = pairs * slots, ctw = 2ull * c.dk * c.n;
    uint64_t* sum = scratch;
    uint64_t* diff = sum + count * ctw;
    uint64_t* moved = diff + count * ctw;
    uint64_t* ks = moved + count * ctw;
    cudaStream_t st = pick(ctx, stream);
    cuda_check(launch_packing_prepare_many(c.P, in, pairs, slots, sum, diff, level, st), "prepare");
    cuda_check(launch_keyswitch(c.P, sum, key_one, 1, count, ks, out, st), "keyswitch");
    cuda_check(launch_keyswitch(c.P, diff, key_level, (2u << level) + 1, count, ks, moved, st), "keyswitch");
    cuda_check(launch_add(c.P, out, moved, count * 2 * c.dk, st), "add");
    count_launch(6);
  });
}

int32_t bfvgpu_token_close(bfvgpu_token* t, bfvgpu_cleanup* cleanup) {
  if (!t) return BFVGPU_E_ARGUMENT;
  const bfvgpu_cleanup c = t->h.release();
  if (cleanup) *cleanup = c;
  return BFVGPU_OK;
}
int32_t bfvgpu_token_release(bfvgpu_token* t) {
  if (!t) return BFVGPU_OK;
  t->h.release();
  delete t;
  return BFVGPU_OK;
}

}  // extern "C"

// ---- library-internal hooks (ctx_internal.h) ---------------------------------------------
namespace bfvgpu {
const DevParams* internal_params(const bfvgpu_ctx* ctx, int* device, cudaStream_t* stream) {
  if (!ctx) return nullptr;
  if (device) *device = ctx->c.device;
  if (stream) *stream = ctx->c.stream;
  return &ctx->c.P;
}
void internal_set_error(const std::string& what) { g_last_error = what; }
void internal_count_launch(uint64_t n) { count_launch(n); }
uint64_t internal_first_prime(const bfvgpu_ctx* ctx) { return ctx && !ctx->c.q.empty() ? ctx->c.q[0] : 0; }
}  // namespace bfvgpu
