"""GPU parity of the 3-bit metadata codec and the 3-bit-metadata GEMM.

Pack/unpack must be bit-exact against the oracle restatement of
``metadata_decode/codec.cu``; the device decoders are checked exhaustively
over all 2^24 code words against the reference's truth tables
(``decoder_dependency/pair.cu:11-30``); the 3-bit GEMM must equal the 4-bit
GEMM bit for bit (same arithmetic, only the metadata encoding differs) --
the reference's own pass rule (``metadata_decode/smoke.py:17-39``).
"""
import os

import numpy as np
import pytest
import torch

import marlin24_oracle as O
from conftest import GOLDEN, golden_cases
from problems import REL_FRO_TOL, REL_MAE_TOL, activations, errors, quantized_problem, random_packed_problem

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_pack_unpack_bit_exact_on_reference_metadata():
    from csed499ii_b200 import metadata_decode as md

    for name in golden_cases():
        meta = np.load(os.path.join(GOLDEN, name))["meta"]
        packed = md.pack(torch.from_numpy(meta).to(DEV))
        ref, err = O.meta3_pack(meta)
        assert err == 0
        assert np.array_equal(packed.cpu().numpy(), ref)
        restored = md.unpack(packed)
        assert torch.equal(restored.cpu(), torch.from_numpy(meta.reshape(-1)))


def _reference_codec():
    """The reference's own codec (metadata_decode/codec.cu), compiled from its
    source by oracle/build_ref.py into oracle/_ref/ (a torch extension)."""
    import glob
    import importlib.machinery
    import importlib.util

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    found = sorted(glob.glob(os.path.join(root, "oracle", "_ref", "ref_codec*.so")))
    if not found:
        pytest.skip("reference codec not built (oracle/build_ref.py needs the reference checkout)")
    loader = importlib.machinery.ExtensionFileLoader("ref_codec", found[0])
    spec = importlib.util.spec_from_loader("ref_codec", loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def _legal_meta(n_int16, seed):
    rng = np.random.default_rng(seed)
    nib = rng.choice(np.array([0x4, 0x8, 0x9, 0xC, 0xD, 0xE], dtype=np.uint16), size=(n_int16, 4))
    return (nib[:, 0] | (nib[:, 1] << 4) | (nib[:, 2] << 8) | (nib[:, 3] << 12)).astype(np.uint16).view(np.int16)


def test_pack_bytes_equal_reference_codec():
    """The packed 3-bit words are the reference codec's bytes, word for word
    (not only a round trip of this library's own pack/unpack): on every golden
    fixture's metadata and on one full 4096 x 4096 layer; and each side's
    unpack inverts the other's pack (codec.cu:18-41, smoke.py:17-18)."""
    from csed499ii_b200 import metadata_decode as md

    ref = _reference_codec()
    metas = [np.load(os.path.join(GOLDEN, name))["meta"].reshape(-1) for name in golden_cases()]
    metas.append(_legal_meta(4096 * 4096 // 16, seed=5))
    for meta in metas:
        t = torch.from_numpy(np.ascontiguousarray(meta)).to(DEV)
        ours = md.pack(t)
        theirs = ref.pack(t)
        torch.cuda.synchronize()
        assert theirs.dtype == torch.int32 and torch.equal(ours, theirs)
        assert torch.equal(md.unpack(theirs).view(-1), t)
        assert torch.equal(ref.unpack(ours).view(-1), t)


def test_pack_rejects_illegal_nibbles():
    from csed499ii_b200 import metadata_decode as md

    meta = torch.full((256,), 0x4444, dtype=torch.int16, device=DEV)
    meta[3] = 0x4F44
    with pytest.raises(RuntimeError, match="unsupported 2:4 nibbles"):
        md.pack(meta)
    with pytest.raises(RuntimeError, match="multiple of 256 bytes"):
        md.pack(meta[:100])
    with pytest.raises(RuntimeError, match="expected compressed metadata"):
        md.unpack(torch.zeros(47, dtype=torch.int32, device=DEV))


def test_decoders_exhaustive():
    from csed499ii_b200 import metadata_decode as md

    x = np.arange(1 << 24, dtype=np.uint32)
    garbage = ((x * np.uint32(1664525) + np.uint32(1013904223)) & np.uint32(0xFF)) << np.uint32(24)
    xin = torch.from_numpy((x | garbage).view(np.int32)).to(DEV)
    hi, lo = md.decode_words(xin)
    assert np.array_equal(hi.cpu().numpy().view(np.uint32), O.decode24(x, O.DEC_HIGH))
    assert np.array_equal(lo.cpu().numpy().view(np.uint32), O.decode24(x, O.DEC_LOW))


def _gemm(A, B, meta, s, N, meta3, sms=-1):
    import csed499ii_b200 as m
    from csed499ii_b200 import metadata_decode as md

    A_d = torch.from_numpy(A).to(DEV)
    C = torch.zeros((A.shape[0], N), dtype=torch.half, device=DEV)
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    B_d, s_d = torch.from_numpy(B).to(DEV), torch.from_numpy(s).to(DEV)
    meta_d = torch.from_numpy(meta).to(DEV)
    if sms != -1:
        # same SM count for both calls: the same kernel and split-K plan
        m._mul(A_d, B_d, md.pack(meta_d) if meta3 else meta_d, C, s_d, ws, -1, -1, sms, 16,
               3 if meta3 else 4)
    elif meta3:
        md.matmul(A_d, B_d, md.pack(meta_d), C, s_d, ws)
    else:
        m.mul_2_4(A_d, B_d, meta_d, C, s_d, ws)
    torch.cuda.synchronize()
    return C


# The 3-bit decoding is exact: the same kernel gives bit-identical results
# from 3-bit and 4-bit metadata.  At M = 64 a 4-bit call on all SMs runs the
# CTA-pair tensor-core kernel (3-bit metadata has no such path), so that case
# pins both calls to the decode kernel with one SM count.
@pytest.mark.parametrize("M,sms", [(1, -1), (16, -1), (64, 16)])
def test_meta3_gemm_equals_meta4_gemm(M, sms):
    W, B, s, meta = quantized_problem(4096, 4096, 128, seed=20261019)
    A = activations(M, 4096)
    c4 = _gemm(A, B, meta, s, 4096, False, sms)
    c3 = _gemm(A, B, meta, s, 4096, True, sms)
    assert torch.equal(c3, c4)
    rel_mae, rel_fro, _ = errors(c3, torch.from_numpy(A).to(DEV).float() @ torch.from_numpy(W).to(DEV).float())
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL


@pytest.mark.parametrize("K,N", [(4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096)])
@pytest.mark.parametrize("M", [1, 16, 64])
def test_meta3_llama7b_shapes(K, N, M):
    W, B, s, meta = random_packed_problem(N, K, 128, seed=11)
    A = activations(M, K)
    sms = 16 if M > 32 else -1  # both calls on the decode kernel (see above)
    c3 = _gemm(A, B, meta, s, N, True, sms)
    c4 = _gemm(A, B, meta, s, N, False, sms)
    assert torch.equal(c3, c4)
    rel_mae, rel_fro, _ = errors(c3, torch.from_numpy(A).to(DEV).float() @ torch.from_numpy(W).to(DEV).float())
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL


# Batches above 64 rows, and 33-64 rows where the pair kernel's tiles fit one
# wave, run the CTA-pair tensor-core kernel, whose dequantising warps decode
# the 3-bit metadata: bit-identical to the same kernel on 4-bit metadata, and
# within the tolerances of the oracle; ragged batches, both scale modes.
@pytest.mark.parametrize("K,N,M,g", [(1024, 1024, 300, 128), (4096, 4096, 64, 128),
                                     (2048, 1536, 1000, -1), (4096, 11008, 200, 128)])
def test_meta3_prefill_pair_kernel(K, N, M, g):
    if g == -1:
        W, B, s, meta = quantized_problem(N, K, -1, seed=K + N)
    else:
        W, B, s, meta = random_packed_problem(N, K, 128, seed=K + N + M)
    A = activations(M, K, seed=M + 6)
    c4 = _gemm(A, B, meta, s, N, False)
    c3 = _gemm(A, B, meta, s, N, True)
    assert torch.equal(c3, c4)
    rel_mae, rel_fro, _ = errors(c3, torch.from_numpy(A).to(DEV).float() @ torch.from_numpy(W).to(DEV).float())
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL


def test_meta3_shape_checks():
    from csed499ii_b200 import metadata_decode as md

    a = torch.zeros((1, 256), dtype=torch.half, device=DEV)
    c = torch.zeros((1, 256), dtype=torch.half, device=DEV)
    bad = torch.zeros(10, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="unsupported compressed metadata shape"):
        md.fetch(a, None, bad, c, None, None)
    with pytest.raises(RuntimeError, match="a must be contiguous CUDA half"):
        md.fetch(a.float(), None, bad, c, None, None)
