"""GPU parity: the CUDA path through the C ABI against the CPU oracle, bit for bit.

Sizes are the BASELINE parameter sets (config 1: n=4096, 3 primes of 36/36/37 bits;
config 2: n=8192, 4 x 50-bit + one 60-bit special prime; ART-002: n=16384, 6+1 x 60-bit)
with batch sizes the oracle finishes in seconds.  Boundary residues follow
IV1/experiments/resident_token_gpu/check_resident.cpp:98 (j%13 in {0,1,2} -> 0, q-1, 1)
and the keyswitch plaintext patterns follow keyswitch_full_gpu/check_switch.cpp:80.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG1 = dict(n=4096, bits=[36, 36, 37], dk=3, special=0, t=65537)
CFG2 = dict(n=8192, bits=[50, 50, 50, 50, 60], dk=4, special=1, t=65537)


@pytest.fixture(scope="module")
def gpu(bfv):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return bfv


def _contexts(bfv, oracle, cfg):
    primes = oracle.coeff_modulus(cfg["n"], cfg["bits"])
    hc = bfv.Context(cfg["n"], primes, cfg["dk"], cfg["special"], cfg["t"], device=0)
    oc = oracle.Ctx(cfg["n"], primes, data_k=cfg["dk"], t=cfg["t"])
    return hc, oc


@pytest.fixture(scope="module")
def art(gpu, oracle):
    return gpu.Context.art002(0), oracle.art002()


@pytest.fixture(scope="module")
def cfg1(gpu, oracle):
    return _contexts(gpu, oracle, CFG1)


@pytest.fixture(scope="module")
def cfg2(gpu, oracle):
    return _contexts(gpu, oracle, CFG2)


def boundary(a: np.ndarray, q) -> np.ndarray:
    """check_resident.cpp:98 pattern on [polys][n] with prime of poly i = q[i % len(q)]."""
    a = a.copy()
    n = a.shape[-1]
    j = np.arange(n)
    flat = a.reshape(-1, n)
    for i in range(flat.shape[0]):
        qi = q[i % len(q)]
        flat[i, j % 13 == 0] = 0
        flat[i, j % 13 == 1] = qi - 1
        flat[i, j % 13 == 2] = 1
    return a


# ---- NTT -----------------------------------------------------------------------------------
def test_ntt_batch_config1_forward_inverse(cfg1):
    hc, oc = cfg1
    batches = 19
    data = boundary(oc.uniform(1, batches * 3), oc.primes).reshape(batches, 3, hc.n)
    nb = __import__("bfvgpu").NttBatch(hc, key_level=False, batches=batches)
    fwd = nb.transform(data, inverse=False)
    assert np.array_equal(fwd, oc.ntt(data, prime_count=3))
    back = nb.transform(fwd, inverse=True)
    assert np.array_equal(back, data)
    c = nb.close()
    assert c["closed"] and c["wiped"] == c["freed"] == data.nbytes
    assert nb.close() == c  # idempotent


def test_ntt_device_config1_full_batch(cfg1):
    """The BASELINE config-1 batch: 64 ciphertexts x 2 polys x 3 limbs, in place."""
    import torch
    hc, oc = cfg1
    data = boundary(oc.uniform(2, 384), oc.primes)
    d = torch.from_numpy(data.view(np.int64)).cuda()
    torch.cuda.synchronize()
    hc.ntt_device(d, 384, 3, 0, inverse=False)
    torch.cuda.synchronize()
    got = d.cpu().numpy().view(np.uint64)
    assert np.array_equal(got, oc.ntt(data, prime_count=3, threads=8))
    hc.ntt_device(d, 384, 3, 0, inverse=True)
    torch.cuda.synchronize()
    assert np.array_equal(d.cpu().numpy().view(np.uint64), data)


def test_ntt_art002_key_level(art):
    hc, oc = art
    data = boundary(oc.uniform(3, 2 * 7, prime_count=7), oc.primes).reshape(2, 7, hc.n)
    nb = __import__("bfvgpu").NttBatch(hc, key_level=True, batches=2)
    fwd = nb.transform(data, inverse=False)
    assert np.array_equal(fwd, oc.ntt(data, prime_count=7))
    assert np.array_equal(nb.transform(fwd, inverse=True), data)


def test_ntt_rejects_non_canonical(art):
    import bfvgpu
    hc, oc = art
    nb = bfvgpu.NttBatch(hc, key_level=False, batches=1)
    bad = np.zeros((1, 6, hc.n), dtype=np.uint64)
    bad[0, 2, 5] = oc.primes[2]
    with pytest.raises(bfvgpu.BfvGpuInvalidArgument) as e:
        nb.transform(bad, inverse=False)
    assert e.value.name == "BFVGPU_E_CANONICAL"
    nb.close()
    with pytest.raises(bfvgpu.BfvGpuError):
        nb.transform(np.zeros((1, 6, hc.n), dtype=np.uint64), inverse=False)


# ---- keyswitch ----------------------------------------------------------------------------
def _ks_case(hc, oc, oracle, seed, elts, patterns=True):
    import bfvgpu
    tb = oracle.TestBfv(oc, seed=seed)
    n = oc.n
    plains = []
    if patterns:
        plains.append(np.zeros(n, dtype=np.uint64))
        p1 = np.zeros(n, dtype=np.uint64)
        p1[n - 1] = oc.t - 1
        plains.append(p1)
        plains.append(((np.arange(n, dtype=np.uint64) * 7919 + 123456) % np.uint64(oc.t)).astype(np.uint64))
    cts = np.stack([tb.encrypt(p) for p in plains])
    for elt in elts:
        key = tb.galois_key(elt)
        sw = bfvgpu.Switch(hc, key, elt)
        got = sw.apply_many(cts)
        for i in range(cts.shape[0]):
            exp = oc.keyswitch(cts[i], key, elt)
            assert np.array_equal(got[i], exp), (elt, i)
        # single-ct entry point, and decryption of the switched ciphertext
        one = sw.apply(cts[2])
        assert np.array_equal(one, got[2])
        dec = tb.decrypt(one)
        m = [int(v) for v in plains[2]]
        exp_plain = [0] * n
        for j in range(n):
            d = (j * elt) % (2 * n)
            if d >= n:
                exp_plain[d - n] = (-m[j]) % oc.t
            else:
                exp_plain[d] = m[j]
        assert dec == exp_plain
        c = sw.close()
        assert c["closed"] and c["first_cuda_error"] == 0 and c["wiped"] == c["freed"] > 0


def test_keyswitch_config2(cfg2, oracle):
    hc, oc = cfg2
    _ks_case(hc, oc, oracle, 11, [3, 3 ** 7 % (2 * oc.n), 2 * oc.n - 1])


def test_keyswitch_art002_acyclic_elements(art, oracle):
    hc, oc = art
    # acyclic packing elements of bfv_acyclic_pack.hpp:30: 1 and 2^(l+1)+1 for l in 0..8
    _ks_case(hc, oc, oracle, 12, [1, 3, 2 ** 9 + 1])


def test_keyswitch_random_residues_with_zero_digits(cfg2, oracle):
    """Uniform residues (no decryption structure) incl. zero coefficients in c1, which
    exercise the zero branch of the automorphism's negation."""
    import bfvgpu
    hc, oc = cfg2
    cts = oc.uniform(21, 4 * 2 * 4).reshape(4, 2, 4, oc.n)
    cts[0, 1, :, ::7] = 0
    key = oc.uniform(22, 4 * 2 * 5, prime_count=5).reshape(4, 2, 5, oc.n)
    for elt in (5, 25, 2 * oc.n - 3):
        sw = bfvgpu.Switch(hc, key, elt)
        got = sw.apply_many(cts)
        exp = oc.keyswitch_many(cts, key, [elt], threads=8)[0]
        assert np.array_equal(got, exp)
        sw.close()


def test_keyswitch_device_batch(cfg2):
    """Device-resident batched entry point agrees with the host-buffer object."""
    import torch
    import bfvgpu
    hc, oc = cfg2
    cts = oc.uniform(31, 8 * 2 * 4).reshape(8, 2, 4, oc.n)
    key = oc.uniform(32, 4 * 2 * 5, prime_count=5).reshape(4, 2, 5, oc.n)
    elt = 3 ** 5 % (2 * oc.n)
    d_cts = torch.from_numpy(cts.view(np.int64)).cuda()
    d_key = torch.from_numpy(key.view(np.int64)).cuda()
    scratch = torch.empty(hc.keyswitch_scratch_words(8), dtype=torch.int64, device="cuda")
    out = torch.empty_like(d_cts)
    torch.cuda.synchronize()
    hc.keyswitch_device(d_cts, 8, d_key, elt, scratch, out)
    torch.cuda.synchronize()
    sw = bfvgpu.Switch(hc, key, elt)
    assert np.array_equal(out.cpu().numpy().view(np.uint64), sw.apply_many(cts))


@pytest.mark.parametrize("which", ["cfg2", "art"])
def test_keyswitch_hoisted_device(which, request, oracle):
    """Hoist once, prepare one key per element, rotate: every output equals the oracle's
    reference keyswitch; a ciphertext with zero c1 words takes the exact path."""
    import torch
    hc, oc = request.getfixturevalue(which)
    n, k, dk = oc.n, oc.k, oc.data_k
    count = 5 if which == "cfg2" else 2
    cts = oc.uniform(51, count * 2 * dk).reshape(count, 2, dk, n)
    cts[1, 1, 0, ::9] = 0
    elts = [3, pow(3, 11, 2 * n), 2 * n - 1] if which == "cfg2" else [1, 2 ** 9 + 1]
    d_cts = torch.from_numpy(cts.view(np.int64)).cuda()
    hoisted = torch.empty(hc.keyswitch_hoist_words(count), dtype=torch.int64, device="cuda")
    prepared = torch.empty(hc.keyswitch_prepared_words(), dtype=torch.int64, device="cuda")
    scratch = torch.empty(hc.keyswitch_scratch_words(count), dtype=torch.int64, device="cuda")
    out = torch.empty_like(d_cts)
    out_plain = torch.empty_like(d_cts)
    torch.cuda.synchronize()
    hc.keyswitch_hoist_device(d_cts, count, hoisted)
    for i, elt in enumerate(elts):
        key = oc.uniform(60 + i, dk * 2 * k, prime_count=k).reshape(dk, 2, k, n)
        d_key = torch.from_numpy(key.view(np.int64)).cuda()
        torch.cuda.synchronize()
        hc.keyswitch_prepare_device(d_key, elt, prepared)
        hc.keyswitch_rotate_device(d_cts, count, hoisted, prepared, elt, scratch, out)
        hc.keyswitch_device(d_cts, count, d_key, elt, scratch, out_plain)
        torch.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint64)
        assert np.array_equal(got, out_plain.cpu().numpy().view(np.uint64)), elt
        exp = oc.keyswitch_many(cts, key, [elt], threads=8)[0]
        assert np.array_equal(got, exp), elt


@pytest.mark.parametrize("which", ["cfg2", "art"])
def test_keyswitch_rotate_many_pipelined(which, request, oracle):
    """The software-pipelined rotations (bfvgpu_keyswitch_rotate_many_device: elements + 1
    launches, each data-prime block finishing its keyswitch in shared memory) equal one
    bfvgpu_keyswitch_rotate_device call per element, word for word, and the oracle; with one
    output per element and with a single output buffer every element overwrites."""
    import torch
    hc, oc = request.getfixturevalue(which)
    n, k, dk = oc.n, oc.k, oc.data_k
    count = 6 if which == "cfg2" else 2
    cts = oc.uniform(71, count * 2 * dk).reshape(count, 2, dk, n)
    cts[2 % count, 1, 1, ::7] = 0  # zero c1 words: the exact path
    elts = ([3, pow(3, 5, 2 * n), 2 * n - 1, 9, pow(3, 77, 2 * n)] if which == "cfg2"
            else [1, 2 ** 9 + 1, 2 ** 3 + 1])
    m = len(elts)
    keys = np.stack([oc.uniform(80 + i, dk * 2 * k, prime_count=k).reshape(dk, 2, k, n) for i in range(m)])
    d_cts = torch.from_numpy(cts.view(np.int64)).cuda()
    d_keys = torch.from_numpy(keys.view(np.int64)).cuda()
    hoisted = torch.empty(hc.keyswitch_hoist_words(count), dtype=torch.int64, device="cuda")
    pw = hc.keyswitch_prepared_words()
    prepared = torch.empty(m * pw, dtype=torch.int64, device="cuda")
    scratch = torch.empty(hc.keyswitch_rotate_many_scratch_words(count), dtype=torch.int64, device="cuda")
    outs = [torch.full_like(d_cts, -1) for _ in range(m)]
    shared = torch.full_like(d_cts, -1)
    one = torch.empty_like(d_cts)
    torch.cuda.synchronize()
    hc.keyswitch_hoist_device(d_cts, count, hoisted)
    hc.keyswitch_prepare_device(d_keys, elts, prepared)
    hc.keyswitch_rotate_many_device(d_cts, count, hoisted, prepared, elts, scratch, outs)
    hc.keyswitch_rotate_many_device(d_cts, count, hoisted, prepared, elts, scratch, shared)
    torch.cuda.synchronize()
    assert hc.check() == 0
    for i, elt in enumerate(elts):
        hc.keyswitch_rotate_device(d_cts, count, hoisted, prepared[i * pw:(i + 1) * pw], elt, scratch, one)
        torch.cuda.synchronize()
        assert torch.equal(outs[i], one), elt
        got = outs[i].cpu().numpy().view(np.uint64)
        assert np.array_equal(got, oc.keyswitch_many(cts, keys[i], [elt], threads=8)[0]), elt
    assert torch.equal(shared, outs[-1])


def test_rotations_object(cfg2, oracle):
    """bfvgpu.Rotations (one upload, hoisted digits, every element streamed back) equals
    Switch.apply_many per element and the oracle; a ciphertext with zero c1 words included."""
    import bfvgpu
    hc, oc = cfg2
    n, k, dk = oc.n, oc.k, oc.data_k
    count = 5
    cts = oc.uniform(71, count * 2 * dk).reshape(count, 2, dk, n)
    cts[2, 1, 1, ::7] = 0
    elts = [3, pow(3, 5, 2 * n), 2 * n - 1]
    keys = np.stack([oc.uniform(80 + i, dk * 2 * k, prime_count=k).reshape(dk, 2, k, n) for i in range(len(elts))])
    rot = bfvgpu.Rotations(hc, keys, elts)
    try:
        bad = cts.copy()
        bad[count - 1, 1, dk - 1, n - 1] = oc.primes[dk - 1]  # one residue equal to its prime
        with pytest.raises(bfvgpu.BfvGpuError) as e:
            rot.apply(bad)  # checked on the device after the upload, before any work
        assert e.value.name == "BFVGPU_E_CANONICAL"
        got = rot.apply(cts)  # the object is unaffected by the rejected batch
        again = rot.apply(cts[:2])  # smaller batch on the same object
    finally:
        assert rot.close()["closed"]
    for i, elt in enumerate(elts):
        sw = bfvgpu.Switch(hc, keys[i], elt)
        try:
            ref = sw.apply_many(cts)
        finally:
            sw.close()
        assert np.array_equal(got[i], ref), elt
        assert np.array_equal(again[i], ref[:2]), elt
    assert np.array_equal(got[0], oc.keyswitch_many(cts, keys[0], [elts[0]], threads=8)[0])


def test_packing_pair(art, oracle):
    import bfvgpu
    hc, oc = art
    tb = oracle.TestBfv(oc, seed=41)
    level = 2
    g = (1 << (level + 1)) + 1
    k1 = tb.galois_key(1)
    kg = tb.galois_key(g)
    rng = np.random.default_rng(3)
    L = tb.encrypt(rng.integers(0, 1 << 20, size=oc.n, dtype=np.uint64))
    R = tb.encrypt(rng.integers(0, 1 << 20, size=oc.n, dtype=np.uint64))
    s1 = bfvgpu.Switch(hc, k1, 1)
    sg = bfvgpu.Switch(hc, kg, g)
    got = s1.packing_pair(L, R, sg, level)
    assert np.array_equal(got, oc.packing_pair(L, R, k1, kg, level))
    with pytest.raises(bfvgpu.BfvGpuError):
        sg.packing_pair(L, R, s1, level)  # wrong element order -> E_PACK_PAIR_STATE


# ---- Enc(0), client phase ---------------------------------------------------------------------
def test_enc0(art, oracle):
    import bfvgpu
    hc, oc = art
    tb = oracle.TestBfv(oc, seed=51)
    pz = bfvgpu.PublicZero(hc, tb.pk)
    for _ in range(2):
        s = tb.samples()
        got = pz.encrypt_from_samples(s)
        assert np.array_equal(got, oc.enc0(s, tb.pk))
        assert all(v == 0 for v in tb.decrypt(got)[:64])
    c = pz.close()
    assert c["closed"] and c["wiped"] == c["freed"]


def test_encrypt_many_device(art, oracle):
    """The client's batched encryption equals PublicZero.encrypt_plain per ciphertext and
    decrypts to the plaintexts."""
    import torch
    import bfvgpu
    hc, oc = art
    n, k, dk = oc.n, oc.k, oc.data_k
    tb = oracle.TestBfv(oc, seed=57)
    rng = np.random.default_rng(58)
    cts = 3
    samples = np.stack([tb.samples() for _ in range(cts)])
    plain = rng.integers(0, 1 << 59, size=(cts, n), dtype=np.uint64)
    plain[0, :3] = [0, (1 << 59) - 1, 1]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()
    out = torch.empty((cts, 2, dk, n), dtype=torch.int64, device="cuda")
    scratch = torch.empty(hc.encrypt_many_scratch_words(cts), dtype=torch.int64, device="cuda")
    hc.encrypt_many_device(dev(samples), dev(tb.pk), dev(plain), cts, scratch, out)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint64)
    pz = bfvgpu.PublicZero(hc, tb.pk)
    try:
        for j in range(cts):
            assert np.array_equal(got[j], pz.encrypt(samples[j], plain[j])), j
    finally:
        pz.close()
    assert tb.decrypt(got[0])[:8] == [int(v) for v in plain[0, :8]]


def test_client_phase(art, oracle):
    import bfvgpu
    hc, oc = art
    tb = oracle.TestBfv(oc, seed=61)
    nb = bfvgpu.NttBatch(hc, key_level=False, batches=3)
    nb.bind_client_key(tb.sk_data_ntt())
    c1 = oc.uniform(62, 3 * 6).reshape(3, 6, oc.n)
    got = nb.client_phase(c1)
    for b in range(3):
        assert np.array_equal(got[b], oc.client_phase(c1[b], tb.sk_data_ntt()))
    with pytest.raises(bfvgpu.BfvGpuError):
        nb.bind_client_key(tb.sk_data_ntt())  # E_CLIENT_KEY_STATE


# ---- matrix -----------------------------------------------------------------------------------
def test_matrix_evaluate_and_selective(art, oracle):
    import bfvgpu
    hc, oc = art
    tb = oracle.TestBfv(oc, seed=71)
    rng = np.random.default_rng(72)
    I = 4
    cts = np.stack([tb.encrypt(rng.integers(0, 1 << 59, size=oc.n, dtype=np.uint64)) for _ in range(I)])
    m = bfvgpu.Matrix(hc, cts)
    ring = rng.integers(0, 1 << 59, size=(I, oc.n), dtype=np.uint64)
    ring[0, :4] = [(1 << 59) - 1, 1 << 58, (1 << 58) - 1, 0]
    cn = oc.matrix_open(cts, threads=8)
    full = m.evaluate(ring)
    assert np.array_equal(full, oc.matrix_evaluate(cn, ring, threads=8))
    targets = [3, 100, 8191, 16383]
    sel = m.evaluate_selective(ring, targets)
    assert np.array_equal(sel, oc.matrix_evaluate(cn, ring, targets=targets, threads=8))
    for bad in ([], [5, 5], [16384], list(range(513))):
        with pytest.raises(bfvgpu.BfvGpuInvalidArgument):
            m.evaluate_selective(ring, bad)
    bad_ring = ring.copy()
    bad_ring[1, 7] = 1 << 59
    with pytest.raises(bfvgpu.BfvGpuInvalidArgument) as e:
        m.evaluate(bad_ring)
    assert e.value.name == "BFVGPU_E_RING"
    c = m.close()
    assert c["closed"] and c["wiped"] == c["freed"] and c["first_cuda_error"] == 0
    assert m.close() == c
    with pytest.raises(bfvgpu.BfvGpuInvalidArgument):
        m.evaluate(ring)  # closed: MATRIX_GPU_SHAPE like the reference


def test_matrix_groups_mask_enc0_crt(art, oracle):
    import bfvgpu
    hc, oc = art
    tb = oracle.TestBfv(oc, seed=81)
    rng = np.random.default_rng(82)
    I, G = 3, 3
    cts = np.stack([tb.encrypt(rng.integers(0, 1 << 59, size=oc.n, dtype=np.uint64)) for _ in range(I)])
    m = bfvgpu.Matrix(hc, cts)
    m.bind_public_key(tb.pk)
    ring = rng.integers(0, 1 << 59, size=(G, I, oc.n), dtype=np.uint64)
    mask = rng.integers(0, 1 << 59, size=(G, oc.n), dtype=np.uint64)
    samples = np.stack([tb.samples() for _ in range(G)])
    targets = [[0, 5, 16383], list(range(7, 7 + 512 * 31, 31)), [9]]
    c1, c0, crt = m.evaluate_groups(ring, targets, mask=mask, samples=samples, crt=True)
    cn = oc.matrix_open(cts, threads=8)
    for g in range(G):
        e = oc.matrix_evaluate(cn, ring[g], threads=8)
        e[0] = oc.sub_plain(e[0], mask[g])
        e = oc.add(e, oc.enc0(samples[g], tb.pk))
        assert np.array_equal(c1[g], e[1])
        for i, t in enumerate(targets[g]):
            assert np.array_equal(c0[g, :, i], e[0][:, t])
            v = sum(int(crt[g, i, l]) << (64 * l) for l in range(6))
            assert v == oracle.crt(e[0][:, t], oc.primes[:6])


@pytest.mark.parametrize("tiles,path", [(3, 0), (9, 0), (9, 1), (3, 2), (9, 2)])
def test_matrix_tiles_device(art, oracle, tiles, path):
    """Layer pipeline through bfvgpu_matrix_tiles_device (tiles in launches of 8/2/1; path 0
    takes tcgen05 for the 8-tile launch and the TMA-staged CUDA-core product for the rest,
    path 1 the TMA-staged CUDA-core product only, path 2 the CUDA-core product with
    per-thread asynchronous-copy staging) against the oracle's per-tile evaluate + sub_plain
    + Enc(0); also without Enc(0), and without mask and Enc(0)."""
    import torch
    hc, oc = art
    n, k, dk = oc.n, oc.k, oc.data_k
    tb = oracle.TestBfv(oc, seed=90 + tiles)
    rng = np.random.default_rng(tiles)
    I, G = 2, 2
    cts = np.stack([np.stack([tb.encrypt(rng.integers(0, 1 << 59, size=n, dtype=np.uint64)) for _ in range(I)])
                    for _ in range(tiles)])
    ring = rng.integers(0, 1 << 59, size=(G, I, n), dtype=np.uint64)
    ring[0, 0, :4] = [(1 << 59) - 1, 1 << 58, (1 << 58) - 1, 0]
    masks = rng.integers(0, 1 << 59, size=(tiles, G, n), dtype=np.uint64)
    samples = np.stack([np.stack([tb.samples() for _ in range(G)]) for _ in range(tiles)])
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()
    d_in, d_ring, d_masks, d_samples, d_pk = dev(cts), dev(ring), dev(masks), dev(samples), dev(tb.pk)
    w = torch.empty((G, I, dk, n), dtype=torch.int64, device="cuda")
    scratch = torch.empty(hc.matrix_tiles_scratch_words(tiles, G), dtype=torch.int64, device="cuda")
    out = torch.empty((tiles, G, 2, dk, n), dtype=torch.int64, device="cuda")
    plain, masked = torch.empty_like(out), torch.empty_like(out)
    torch.cuda.synchronize()
    hc.set_product_path(path)
    try:
        hc.matrix_tiles_inputs_device(d_in, tiles * I)  # in place
        hc.weights_ntt_device(d_ring, G * I, w)
        pk_prep = torch.empty((2, k, n, 2), dtype=torch.int64, device="cuda")
        hc.matrix_tiles_prepare_pk_device(d_pk, pk_prep)
        hc.matrix_tiles_device(d_in, tiles, I, w, G, out, masks=d_masks, samples=d_samples, pk_prep=pk_prep,
                               scratch=scratch)
        hc.matrix_tiles_device(d_in, tiles, I, w, G, plain)
        hc.matrix_tiles_device(d_in, tiles, I, w, G, masked, masks=d_masks, scratch=scratch)
        # the same call in two parts (protection prepared ahead, then product + transform)
        split = torch.empty_like(out)
        scratch2 = torch.empty_like(scratch)
        hc.matrix_tiles_protect_device(tiles, G, scratch2, masks=d_masks, samples=d_samples, pk_prep=pk_prep)
        hc.matrix_tiles_prepared_device(d_in, tiles, I, w, G, split, enc0=True, masked=True, pk_prep=pk_prep,
                                        scratch=scratch2)
        assert hc.check() == 0
        assert torch.equal(split, out)
    finally:
        hc.set_product_path(0)
    got, got_plain = out.cpu().numpy().view(np.uint64), plain.cpu().numpy().view(np.uint64)
    got_masked = masked.cpu().numpy().view(np.uint64)
    for t in range(tiles):
        cn = oc.matrix_open(cts[t], threads=8)
        for g in range(G):
            e = oc.matrix_evaluate(cn, ring[g], threads=8)
            assert np.array_equal(got_plain[t, g], e), (t, g)
            e[0] = oc.sub_plain(e[0], masks[t, g])
            assert np.array_equal(got_masked[t, g], e), (t, g)
            e = oc.add(e, oc.enc0(samples[t, g], tb.pk))
            assert np.array_equal(got[t, g], e), (t, g)


def test_matrix_tiles_tensor_core_vs_cuda_core(art, oracle):
    """8 tiles, 40 input blocks (K padded to 64), 33 groups (a partial 32-group chunk): the
    tcgen05 product equals the CUDA-core product on every word, and spot (tile, group)
    pairs equal the oracle."""
    import torch
    hc, oc = art
    n, k, dk = oc.n, oc.k, oc.data_k
    tiles, I, G = 8, 40, 33
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)
    q = torch.tensor(oc.primes[:dk], dtype=torch.int64, device="cuda").view(dk, 1)
    cts = torch.remainder(torch.randint(0, 2 ** 62, (tiles, I, 2, dk, n), dtype=torch.int64, device="cuda",
                                        generator=gen), q)
    cts[0, 0, 0, 0, :64] = q[0] - 1  # boundary residues
    cts[1, 1, 1, 2, :64] = 0
    ring = torch.randint(-127, 128, (G, I, n), dtype=torch.int64, device="cuda", generator=gen) & ((1 << 59) - 1)
    d_in = cts.clone()
    w = torch.empty((G, I, dk, n), dtype=torch.int64, device="cuda")
    out_tc = torch.empty((tiles, G, 2, dk, n), dtype=torch.int64, device="cuda")
    out_cc = torch.empty_like(out_tc)
    hc.matrix_tiles_inputs_device(d_in, tiles * I)
    hc.weights_ntt_device(ring, G * I, w)
    hc.matrix_tiles_device(d_in, tiles, I, w, G, out_tc)
    hc.set_product_path(1)
    try:
        hc.matrix_tiles_device(d_in, tiles, I, w, G, out_cc)
    finally:
        hc.set_product_path(0)
    assert hc.check() == 0
    assert torch.equal(out_tc, out_cc)
    got = out_tc.cpu().numpy().view(np.uint64)
    cts_h = cts.cpu().numpy().view(np.uint64)
    ring_h = ring.cpu().numpy().view(np.uint64)
    for t, g in [(0, 0), (1, 32), (7, 17)]:
        cn = oc.matrix_open(cts_h[t], threads=8)
        assert np.array_equal(got[t, g], oc.matrix_evaluate(cn, ring_h[g], threads=8)), (t, g)


def test_limb_split_equals_one_block_per_limb(art, oracle):
    """At n = 16384 the single-transform kernels split each limb between the two blocks of a
    cluster (the default).  Every kernel that takes that form -- batched forward and inverse
    NTT, weight lift + NTT, client-limb transform, Enc(0) preparation and the protected output
    transform of the tile product -- gives the same words as with one block per limb, and the
    NTT equals the oracle."""
    import torch
    hc, oc = art
    n, k, dk = oc.n, oc.k, oc.data_k
    gen = torch.Generator(device="cuda")
    gen.manual_seed(17)
    q = torch.tensor(oc.primes, dtype=torch.int64, device="cuda")
    res = lambda shape, m: torch.remainder(
        torch.randint(0, 2 ** 62, shape, dtype=torch.int64, device="cuda", generator=gen), q[:m].view(m, 1))
    data = res((5, k, n), k)
    data[0, 0, :3] = torch.tensor([0, 1, oc.primes[0] - 1])
    tiles, I, G = 2, 5, 3
    cts = res((tiles, I, 2, dk, n), dk)
    ring = torch.randint(-(1 << 20), 1 << 20, (G, I, n), dtype=torch.int64, device="cuda", generator=gen) & ((1 << 59) - 1)
    masks = torch.randint(0, 2 ** 59, (tiles, G, n), dtype=torch.int64, device="cuda", generator=gen)
    small = torch.cat([torch.randint(-1, 2, (tiles, G, 1, n), device="cuda", generator=gen),
                       torch.randint(-5, 6, (tiles, G, 2, n), device="cuda", generator=gen)], dim=2)
    samples = torch.remainder(small.unsqueeze(-2), q.view(k, 1)).contiguous()
    pk = res((2, k, n), k)

    def run():
        f = data.clone()
        hc.ntt_device(f, 5 * k, k)
        b = f.clone()
        hc.ntt_device(b, 5 * k, k, inverse=True)
        d_in = cts.clone()
        hc.matrix_tiles_inputs_device(d_in, tiles * I)
        w = torch.empty((G, I, dk, n), dtype=torch.int64, device="cuda")
        hc.weights_ntt_device(ring, G * I, w)
        pk_prep = torch.empty((2, k, n, 2), dtype=torch.int64, device="cuda")
        hc.matrix_tiles_prepare_pk_device(pk, pk_prep)
        scratch = torch.empty(hc.matrix_tiles_scratch_words(tiles, G), dtype=torch.int64, device="cuda")
        out = torch.empty((tiles, G, 2, dk, n), dtype=torch.int64, device="cuda")
        hc.matrix_tiles_device(d_in, tiles, I, w, G, out, masks=masks, samples=samples, pk_prep=pk_prep,
                               scratch=scratch)
        torch.cuda.synchronize()
        return f, b, d_in, w, out

    torch.cuda.synchronize()
    # torch's copies and the library's kernels on one stream (the context's)
    with torch.cuda.stream(torch.cuda.ExternalStream(hc.stream())):
        split = run()
        hc.set_limb_split(False)
        try:
            whole = run()
        finally:
            hc.set_limb_split(True)
    assert hc.check() == 0
    for name, a, b in zip(("ntt", "intt", "inputs", "weights", "tiles"), split, whole):
        assert torch.equal(a, b), name
    assert torch.equal(split[1], data)
    assert np.array_equal(split[0].cpu().numpy().view(np.uint64),
                          oc.ntt(data.cpu().numpy().view(np.uint64).reshape(5 * k, n), prime_count=k).reshape(5, k, n))


def test_matrix_tiles_qkv_full_shape(art, oracle):
    """The benchmark's largest prefill call at full shape: the qkv joint projection of a
    128-token group, 8 tiles x 64 input blocks x 128 output groups (matrix_packing of B = 16,
    K = 1024, O = 4096), int8 weights, with the masks and Enc(0) of every output, on the
    tcgen05 product.  Every output word equals the CUDA-core product's, and spot (tile, group)
    pairs equal the oracle's evaluate + sub_plain + Enc(0) + add."""
    import torch
    hc, oc = art
    n, k, dk = oc.n, oc.k, oc.data_k
    tiles, I, G = 8, 64, 128
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)
    q = torch.tensor(oc.primes, dtype=torch.int64, device="cuda")

    def residues(shape, nprimes, lo=0, hi=None):
        """Values in [lo, hi) (uniform residues when hi is None) reduced per prime (axis -2)."""
        if hi is None:
            raw = torch.randint(0, 2 ** 62, shape, dtype=torch.int64, device="cuda", generator=gen)
        else:
            raw = torch.randint(lo, hi, shape, dtype=torch.int64, device="cuda", generator=gen)
        return torch.remainder(raw, q[:nprimes].view(*([1] * (len(shape) - 2)), nprimes, 1))

    cts = residues((tiles, I, 2, dk, n), dk)
    cts[0, 0, 0, 0, :64] = q[0] - 1
    ring = torch.randint(-127, 128, (G, I, n), dtype=torch.int64, device="cuda", generator=gen) & ((1 << 59) - 1)
    masks = torch.randint(0, 2 ** 59, (tiles, G, n), dtype=torch.int64, device="cuda", generator=gen)
    # Enc(0) randomness as the sampler draws it: ternary u, small e0, e1, each in all k primes
    small = lambda lo, hi: torch.randint(lo, hi, (tiles, G, 1, n), dtype=torch.int64, device="cuda",
                                         generator=gen).expand(tiles, G, k, n)
    samples = torch.stack([torch.remainder(small(lo, hi), q.view(1, 1, k, 1))
                           for lo, hi in ((-1, 2), (-5, 6), (-5, 6))], dim=2).contiguous()
    pk = residues((2, k, n), k)
    d_in = cts.clone()
    w = torch.empty((G, I, dk, n), dtype=torch.int64, device="cuda")
    pk_prep = torch.empty((2, k, n, 2), dtype=torch.int64, device="cuda")
    scratch = torch.empty(hc.matrix_tiles_scratch_words(tiles, G), dtype=torch.int64, device="cuda")
    out_tc = torch.empty((tiles, G, 2, dk, n), dtype=torch.int64, device="cuda")
    out_cc = torch.empty_like(out_tc)
    hc.matrix_tiles_inputs_device(d_in, tiles * I)
    hc.weights_ntt_device(ring, G * I, w)
    hc.matrix_tiles_prepare_pk_device(pk, pk_prep)
    hc.matrix_tiles_device(d_in, tiles, I, w, G, out_tc, masks=masks, samples=samples, pk_prep=pk_prep,
                           scratch=scratch)
    hc.set_product_path(1)
    try:
        hc.matrix_tiles_device(d_in, tiles, I, w, G, out_cc, masks=masks, samples=samples, pk_prep=pk_prep,
                               scratch=scratch)
    finally:
        hc.set_product_path(0)
    assert hc.check() == 0
    assert torch.equal(out_tc, out_cc)
    pk_h = pk.cpu().numpy().view(np.uint64)
    for t, g in [(0, 0), (3, 63), (5, 100), (7, 127)]:
        cn = oc.matrix_open(cts[t].cpu().numpy().view(np.uint64), threads=8)
        e = oc.matrix_evaluate(cn, ring[g].cpu().numpy().view(np.uint64), threads=8)
        e[0] = oc.sub_plain(e[0], masks[t, g].cpu().numpy().view(np.uint64))
        e = oc.add(e, oc.enc0(samples[t, g].cpu().numpy().view(np.uint64), pk_h))
        assert np.array_equal(out_tc[t, g].cpu().numpy().view(np.uint64), e), (t, g)


# ---- resident token ----------------------------------------------------------------------------
def test_token_weights(art, oracle):
    import bfvgpu
    hc, oc = art
    rng = np.random.default_rng(91)
    slots = 1
    cts = oc.uniform(92, slots * 19 * 2 * 6).reshape(slots, 19, 2, 6, oc.n)
    cts = boundary(cts.reshape(-1, oc.n), oc.primes[:6]).reshape(cts.shape)
    tw = bfvgpu.TokenWeights(hc, cts)
    bound = 1 << 20
    for case in range(2):
        if case == 0:
            vals = np.array([0, 1, -1, bound, -bound, bound - 1, -(bound - 1)], dtype=np.int64)
            ring = (vals[np.arange(19 * 8192) % 7] & ((1 << 59) - 1)).astype(np.uint64)
        else:
            ring = (rng.integers(-bound, bound + 1, size=19 * 8192) & ((1 << 59) - 1)).astype(np.uint64)
        local = rng.integers(0, 1 << 59, size=slots, dtype=np.uint64)
        got = tw.evaluate_finished(ring, local)
        inputs_ntt = np.stack([oc.ntt(cts[s].reshape(-1, oc.n), prime_count=6).reshape(19, 2, 6, oc.n)
                               for s in range(slots)], axis=1)  # [19][slots][2][6][n]
        scaled = np.array([oc.scale_plain(int(v)) for v in local], dtype=np.uint64)
        exp = oc.token_evaluate(inputs_ntt, slots, ring, scaled)
        assert np.array_equal(got, exp), case
    bad = np.zeros(19 * 8192, dtype=np.uint64)
    bad[0] = bound + 1
    with pytest.raises(bfvgpu.BfvGpuInvalidArgument) as e:
        tw.evaluate_finished(bad, np.zeros(slots, dtype=np.uint64))
    assert e.value.name == "BFVGPU_E_BOUND"
    c = tw.close()
    assert c["closed"] and c["wiped"] == c["freed"]


@pytest.mark.parametrize("slots,coords", [(2, 8), (1, 64)])
def test_token_tile_batched(art, oracle, slots, coords):
    """Raw token products of `coords` coordinates in one batched call equal TokenWeights, one
    coordinate at a time; the level-batched packing tree over them (log2 coords levels: 3, and
    6 at 64 coordinates) equals the reference's binary-counter stack of pairwise merges
    (Switch.packing_pair, itself checked against the oracle)."""
    import torch
    import bfvgpu
    hc, oc = art
    n, dk, k = oc.n, oc.data_k, oc.k
    rng = np.random.default_rng(95 + coords)
    bound = 1 << 20
    cts = oc.uniform(96, slots * 19 * 2 * dk).reshape(slots, 19, 2, dk, n)
    tw = bfvgpu.TokenWeights(hc, cts)
    ring = (rng.integers(-bound, bound + 1, size=(coords, 19 * 8192)) & ((1 << 59) - 1)).astype(np.uint64)
    local = rng.integers(0, 1 << 59, size=(coords, slots), dtype=np.uint64)
    try:
        ref = np.stack([tw.evaluate_finished(ring[j], local[j]) for j in range(coords)])  # [coords][slots][2][dk][n]
    finally:
        tw.close()
    inputs_ntt = np.stack([oc.ntt(cts[s].reshape(-1, n), prime_count=dk).reshape(19, 2, dk, n)
                           for s in range(slots)], axis=1)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()
    d_in, d_ring, d_local = dev(inputs_ntt), dev(ring), dev(local)
    scratch = torch.empty(hc.token_many_scratch_words(coords, slots), dtype=torch.int64, device="cuda")
    raw = torch.empty((coords, slots, 2, dk, n), dtype=torch.int64, device="cuda")
    hc.token_evaluate_many_device(d_in, slots, d_ring, coords, d_local, scratch, raw)
    torch.cuda.synchronize()
    assert np.array_equal(raw.cpu().numpy().view(np.uint64), ref)
    # packing tree: level l merges pairs of 2^l-coordinate blocks with the level's two keys
    levels = coords.bit_length() - 1
    key_one = [oc.uniform(200 + l, dk * 2 * k, prime_count=k).reshape(dk, 2, k, n) for l in range(levels)]
    key_lev = [oc.uniform(300 + l, dk * 2 * k, prime_count=k).reshape(dk, 2, k, n) for l in range(levels)]
    # torch allocates and frees on the context's stream, so no buffer is reused while a
    # level's kernels still read it
    with torch.cuda.stream(torch.cuda.ExternalStream(hc.stream())):
        d_one, d_lev = [dev(x) for x in key_one], [dev(x) for x in key_lev]
        cur, count = raw, coords
        scr = torch.empty(hc.packing_level_scratch_words((coords // 2) * slots), dtype=torch.int64, device="cuda")
        for l in range(levels):
            pairs = count // 2
            out = torch.empty((pairs, slots, 2, dk, n), dtype=torch.int64, device="cuda")
            hc.packing_level_device(cur, pairs, slots, l, d_one[l], d_lev[l], scr, out)
            cur, count = out, pairs
    torch.cuda.synchronize()
    got = cur[0].cpu().numpy().view(np.uint64)
    sw = [(bfvgpu.Switch(hc, key_one[l], 1), bfvgpu.Switch(hc, key_lev[l], (2 << l) + 1)) for l in range(levels)]
    try:
        for s in range(slots):
            stack = [None] * (levels + 1)
            for j in range(coords):
                current, l = ref[j, s], 0
                while stack[l] is not None:
                    current = sw[l][0].packing_pair(stack[l], current, sw[l][1], l)
                    stack[l], l = None, l + 1
                stack[l] = current
            assert np.array_equal(got[s], stack[levels]), s
    finally:
        for a, b in sw:
            a.close()
            b.close()
