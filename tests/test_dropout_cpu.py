"""CPU checks of the dropout support: the Philox4x32-10 oracle against the published
known-answer vectors, the keep-bit packing, the modules' draw order and shapes against the
reference's definition (src/genie_tk/pair_transform.py:26-61), and the C ABI's argument
validation of the dropout entry points. No kernel is launched here."""

import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import dropout_oracle as D

# Philox4x32-10 known-answer vectors published with the generator (Salmon et al., SC'11,
# Random123 distribution): (counter, key) -> output.
PHILOX_KAT = [
    ((0x00000000, 0x00000000, 0x00000000, 0x00000000), (0x00000000, 0x00000000),
     (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF), (0xFFFFFFFF, 0xFFFFFFFF),
     (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,expected", PHILOX_KAT)
def test_philox_oracle_known_answers(ctr, key, expected):
    out = D.philox4x32_10(np.array(ctr, dtype=np.uint32), np.array(key, dtype=np.uint32))
    assert tuple(int(x) for x in out) == expected


def test_philox_oracle_is_vectorised_consistently():
    ctrs = np.array([c for c, _, _ in PHILOX_KAT], dtype=np.uint32)
    keys = np.array([k for _, k, _ in PHILOX_KAT], dtype=np.uint32)
    out = D.philox4x32_10(ctrs, keys)
    assert [tuple(int(x) for x in row) for row in out] == [e for _, _, e in PHILOX_KAT]


@pytest.mark.parametrize("p", [0.0, 0.1, 0.25, 0.5, 0.9])
def test_keep_bits_rate_and_determinism(p):
    bits = D.keep_bits_philox(seed=42, offset=3, p=p, n_vectors=4096)
    keep = D.unpack_keep(bits)
    rate = keep.mean()
    # 524,288 Bernoulli draws: 6 sigma is below 0.5% of the rate
    assert abs(rate - (1 - p)) < 6 * np.sqrt(p * (1 - p) / keep.size) + 1e-12
    assert np.array_equal(bits, D.keep_bits_philox(seed=42, offset=3, p=p, n_vectors=4096))
    if p > 0:
        assert not np.array_equal(bits, D.keep_bits_philox(seed=42, offset=4, p=p, n_vectors=4096))
        assert not np.array_equal(bits, D.keep_bits_philox(seed=43, offset=3, p=p, n_vectors=4096))
    # a prefix of a longer draw is the shorter draw (the counter is the vector index)
    assert np.array_equal(bits[:100], D.keep_bits_philox(seed=42, offset=3, p=p, n_vectors=100))


def test_keep_bits_channels_are_independent():
    keep = D.unpack_keep(D.keep_bits_philox(seed=7, offset=0, p=0.5, n_vectors=8192)).astype(np.float64)
    corr = np.corrcoef(keep[:, :8].T)
    off = corr[~np.eye(8, dtype=bool)]
    assert np.abs(off).max() < 0.05


def test_pack_unpack_round_trip():
    rng = np.random.default_rng(0)
    keep = rng.random((33, 128)) > 0.4
    bits = D.pack_keep(keep)
    assert bits.dtype == np.uint32 and bits.shape == (33, 4)
    assert np.array_equal(D.unpack_keep(bits), keep)
    # bit c % 32 of word c // 32
    one = np.zeros((1, 128), dtype=bool)
    one[0, 37] = True
    assert D.pack_keep(one).tolist() == [[0, 1 << 5, 0, 0]]


def test_multipliers_from_bits_shapes():
    bits = D.keep_bits_philox(1, 0, 0.25, 2 * 5)
    row = D.multipliers_from_bits(bits, 4 / 3, 2, 5, rowwise=True)
    col = D.multipliers_from_bits(bits, 4 / 3, 2, 5, rowwise=False)
    assert tuple(row.shape) == (2, 1, 5, 128) and tuple(col.shape) == (2, 5, 1, 128)
    assert set(np.unique(row.numpy()).tolist()) <= {0.0, np.float32(4 / 3)}


@pytest.mark.parametrize("cls_name,shared_dim", [("DropoutRowwise", -3), ("DropoutColumnwise", -2)])
def test_dropout_modules_follow_the_reference_definition(cls_name, shared_dim):
    """forward(x) = x * nn.Dropout(p)(ones with the shared axis collapsed), drawing from the
    generator exactly like the reference module (pair_transform.py:33-42, :52-61)."""
    from genie_tk import pair_transform
    x = torch.randn(2, 6, 6, 128)
    mod = getattr(pair_transform, cls_name)(0.25).train()
    torch.manual_seed(11)
    got = mod(x)
    torch.manual_seed(11)
    shape = list(x.shape)
    shape[shared_dim] = 1
    ref = x * torch.nn.Dropout(0.25)(x.new_ones(shape))
    assert torch.equal(got, ref)
    mod.eval()
    assert mod(x) is x
    assert mod.keep_mask(x.shape, x.dtype, x.device) is None


def test_keep_mask_requires_cuda_in_training_mode():
    from genie_tk import pair_transform
    mod = pair_transform.DropoutRowwise(0.25).train()
    with pytest.raises(RuntimeError, match="CUDA"):
        mod.keep_mask((1, 4, 4, 128), torch.float32, torch.device("cpu"))
    assert pair_transform.DropoutRowwise(0.0).train().keep_mask((1, 4, 4, 128), torch.float32,
                                                                torch.device("cpu")) is None


@pytest.fixture(scope="module")
def lib():
    import genie_tk._lib as L
    if not os.path.exists(L.LIB_PATH):
        import __graft_entry__ as g
        g.build()
    return L.load()


def test_dropout_entry_points_validate_arguments(lib):
    import genie_tk._lib as L
    fake = 1 << 20  # never dereferenced: every call below fails validation first
    assert lib.gtk_dropout_keep_bits_philox(1, 0, 1.0, 4, fake, None) == -1
    assert lib.gtk_dropout_keep_bits_philox(1, 0, -0.1, 4, fake, None) == -1
    assert lib.gtk_dropout_keep_bits_philox(1, 0, 0.25, 0, fake, None) == -1
    assert lib.gtk_dropout_keep_bits_philox(1, 0, 0.25, 4, None, None) == -1
    assert lib.gtk_dropout_pack_keep_bits(None, 4, fake, None) == -1
    assert lib.gtk_dropout_pack_keep_bits(fake, 0, fake, None) == -1

    def trimul(d):
        return lib.gtk_trimul_forward_dropout(1, fake, None, fake, fake, 1, ctypes.byref(d), fake, 1 << 40, 1, 64,
                                              128, 128, None, None)

    def triatt(d):
        return lib.gtk_triatt_forward_dropout(0, fake, None, fake, fake, 1, ctypes.byref(d), fake, 1 << 40, 1, 64,
                                              128, 128, 4, 1e9, None, None)

    for call in (trimul, triatt):
        assert call(L.Dropout(None, 1.0, 1)) == -1                      # no keep bits
        assert call(L.Dropout(fake + 4, 1.0, 1)) == -3                  # misaligned
        assert call(L.Dropout(fake, float("nan"), 1)) == -1             # bad scale
        assert call(L.Dropout(fake, -1.0, 0)) == -1
        msg = lib.gtk_last_error_string().decode()
        assert "dropout" in msg


def test_multipliers_from_bits_with_channel_groups():
    """A C-channel mask is ceil(C / 128) consecutive 128-bit groups per (b, residue): group g
    of vector (b, t) holds channels 128 g .. 128 g + 127."""
    rng = np.random.default_rng(5)
    B, N, C = 2, 3, 200
    G = (C + 127) // 128
    keep = rng.random((B * N, G * 128)) > 0.3
    keep[:, C:] = True  # channels past C do not exist
    bits = D.pack_keep(keep.reshape(-1, 128))            # [B * N * G, 4]
    assert bits.shape == (B * N * G, 4)
    m = D.multipliers_from_bits(bits, 2.0, B, N, rowwise=False)
    assert tuple(m.shape) == (B, N, 1, G * 128)
    want = torch.from_numpy(keep.astype(np.float32) * 2.0).reshape(B, N, 1, G * 128)
    assert torch.equal(m, want)
    # the same bits read as int32 [B, N, 4 G] (the library's keep_bits tensor) unpack alike
    kb = bits.view(np.int32).reshape(B, N, 4 * G)
    m2 = D.multipliers_from_bits(kb.view(np.uint32).reshape(-1, 4), 2.0, B, N, rowwise=True)
    assert tuple(m2.shape) == (B, 1, N, G * 128) and torch.equal(m2[:, 0], want[:, :, 0])
