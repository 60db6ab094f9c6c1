"""CPU checks of the C ABI library: it loads, exports every symbol the public header
declares, and its host-only entry points (sizes, layouts, argument validation) behave.
No kernel is launched here."""

import ctypes
import os
import re

import pytest

import genie_tk._lib as L

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "genie_tk_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"GTK_API\s+[\w\s\*]+?\b(gtk_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    import genie_tk._lib as L
    if not os.path.exists(L.LIB_PATH):
        import __graft_entry__ as g
        g.build()
    return L.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ("gtk_trimul_forward", "gtk_triatt_forward", "gtk_trimul_contract", "gtk_triatt_core",
                 "gtk_last_error_string", "gtk_version"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    missing = [s for s in declared_symbols() if getattr(lib, s, None) is None]
    assert not missing, missing


def test_every_declared_symbol_has_a_ctypes_signature():
    import genie_tk._lib as L
    missing = [s for s in declared_symbols() if s not in L.exported_names()]
    assert not missing, missing


def test_host_queries(lib):
    assert lib.gtk_version() >= 100
    assert lib.gtk_trimul_packed_bytes(128, 128) > 0
    assert lib.gtk_triatt_packed_bytes(128, 128, 4) > 0
    # the general-shape path: any channel count up to 512, head_dim up to 64
    for cz, c in ((64, 128), (64, 32), (32, 16), (128, 64), (96, 48)):
        assert lib.gtk_trimul_packed_bytes(cz, c) > 0
        assert lib.gtk_trimul_workspace_bytes(1, 10, cz, c) > 0
    for cin, c, h in ((128, 32, 4), (64, 32, 4), (32, 16, 2), (128, 16, 4), (128, 128, 8), (48, 36, 3)):
        assert lib.gtk_triatt_packed_bytes(cin, c, h) > 0
        assert lib.gtk_triatt_workspace_bytes(1, 10, cin, c, h) > 0
    assert lib.gtk_trimul_packed_bytes(1024, 128) == 0
    # c_z = 128 with a narrower hidden width packs into the tuned 128-channel layout
    assert lib.gtk_trimul_packed_bytes(128, 64) == lib.gtk_trimul_packed_bytes(128, 128)
    assert lib.gtk_trimul_workspace_bytes(1, 10, 128, 1) == lib.gtk_trimul_workspace_bytes(1, 10, 128, 128)
    assert lib.gtk_triatt_packed_bytes(128, 128, 3) == 0    # c_hidden not a multiple of heads
    assert lib.gtk_triatt_packed_bytes(128, 256, 2) == 0    # head_dim 128 > 64
    assert lib.gtk_transition_packed_bytes(64, 4) > 0 and lib.gtk_transition_packed_bytes(128, 2) > 0
    assert [lib.gtk_plane_pitch(n) for n in (1, 8, 10, 1024)] == [8, 8, 16, 1024]
    w1 = lib.gtk_trimul_workspace_bytes(1, 100, 128, 128)
    w2 = lib.gtk_trimul_workspace_bytes(1, 200, 128, 128)
    assert 0 < w1 < w2 and w1 % 256 == 0
    assert lib.gtk_triatt_workspace_bytes(2, 64, 128, 128, 4) > lib.gtk_triatt_workspace_bytes(1, 64, 128, 128, 4)


def test_triatt_workspace_layout(lib):
    B, N = 2, 100
    offs = (ctypes.c_int64 * 7)()
    assert lib.gtk_triatt_workspace_offsets(B, N, N, offs) == 0
    o = list(offs)
    pair16 = B * N * N * 128 * 2
    assert o[0] == 0 and all(x % 256 == 0 for x in o)
    assert all(o[k + 1] - o[k] >= pair16 for k in range(5))
    total = lib.gtk_triatt_workspace_bytes(B, N, 128, 128, 4)
    assert o[6] == total
    assert total - o[5] >= N * B * 4 * lib.gtk_plane_pitch(N) * 2
    # a shard of 25 rows: per-pair intermediates shrink, the bias still covers all N rows
    assert lib.gtk_triatt_workspace_offsets(B, 25, N, offs) == 0
    s = list(offs)
    assert s[1] - s[0] >= B * 25 * N * 128 * 2 and s[1] < o[1]
    assert s[6] - s[5] >= N * B * 4 * lib.gtk_plane_pitch(N) * 2
    assert lib.gtk_triatt_workspace_offsets(B, N + 1, N, offs) == -1


def test_row_shards_are_starting_orientation_only(lib):
    P = ctypes.c_void_p
    rc = lib.gtk_triatt_project(0, P(256), P(256), P(256), 1, 32, 64, 0, None, None)
    assert rc == -2 and b"ending" in lib.gtk_last_error_string()
    rc = lib.gtk_triatt_core(1, None, P(256), 1, 32, 64, 40, 1e9, None, None)
    assert rc == -1 and b"row0" in lib.gtk_last_error_string()


def test_unsupported_shapes_fail_before_touching_the_device(lib):
    rc = lib.gtk_trimul_forward(1, None, None, None, None, 0, None, 0, 1, 16, 1024, 128, None, None)
    assert rc == L.GTK_ERR_UNSUPPORTED
    assert b"c_z" in lib.gtk_last_error_string()
    rc = lib.gtk_triatt_forward(1, None, None, None, None, 0, None, 0, 1, 16, 128, 128, 3, 1e9, None, None)
    assert rc == L.GTK_ERR_UNSUPPORTED
    assert b"heads" in lib.gtk_last_error_string()
    rc = lib.gtk_triatt_forward(1, None, None, None, None, 0, None, 0, 1, 16, 128, 256, 2, 1e9, None, None)
    assert rc == L.GTK_ERR_UNSUPPORTED and b"head_dim" in lib.gtk_last_error_string()
    # the no-alloc entry point keeps to the tuned shape
    rc = lib.gtk_trimul_forward_noalloc(1, None, None, None, None, 0, 1, 16, 64, 64, None, None)
    assert rc == L.GTK_ERR_UNSUPPORTED


def test_general_path_validates_before_touching_the_device(lib):
    # a NULL pair tensor, then a short workspace, at a general shape
    rc = lib.gtk_trimul_forward(1, None, None, None, None, 0, None, 0, 1, 16, 64, 32, None, None)
    assert rc == L.GTK_ERR_INVALID_ARG
    p = ctypes.c_void_p(1 << 20)
    rc = lib.gtk_trimul_forward(1, p, None, p, p, 0, p, 256, 1, 16, 64, 32, None, None)
    assert rc == L.GTK_ERR_WORKSPACE and b"workspace" in lib.gtk_last_error_string()
    rc = lib.gtk_triatt_forward(0, p, None, p, p, 0, p, 256, 1, 16, 128, 32, 4, 1e9, None, None)
    assert rc == L.GTK_ERR_WORKSPACE
    rc = lib.gtk_transition_forward(p, None, p, p, 1, p, 256, 1, 16, 64, 4, None, None)
    assert rc == L.GTK_ERR_WORKSPACE


def test_invalid_arguments_are_rejected(lib):
    # workspace too small is detected from the sizes alone
    rc = lib.gtk_trimul_forward(1, None, None, None, None, 0, None, 0, 1, 16, 128, 128, None, None)
    assert rc == L.GTK_ERR_WORKSPACE
    # a NULL pair tensor is rejected before any launch
    rc = lib.gtk_trimul_project(None, None, None, None, None, 16, 1, 16, 16, None, None)
    assert rc == -1
    # pitches must be multiples of 8
    rc = lib.gtk_trimul_contract(1, ctypes.c_void_p(256), ctypes.c_void_p(256), ctypes.c_void_p(256), 1, 1, 16, 16,
                                 16, 12, 16, 16, 1.0, None, None)
    assert rc == -3
    # the contraction output scale must be positive for the finish stage
    rc = lib.gtk_trimul_finish(ctypes.c_void_p(256), ctypes.c_void_p(256), 16, 0.0, ctypes.c_void_p(256),
                               ctypes.c_void_p(256), 0, 1, 16, 16, None, None)
    assert rc == -1


def test_attention_and_linear_entry_points_validate_before_touching_the_device(lib):
    p = ctypes.c_void_p(1 << 20)
    # head_dim beyond 64, then a zero output-gradient scale, then bad sizes
    rc = lib.gtk_attn_core_forward(p, p, p, p, None, 1, 16, 2, 65, 1e9, p, p, None)
    assert rc == L.GTK_ERR_UNSUPPORTED and b"head_dim" in lib.gtk_last_error_string()
    rc = lib.gtk_attn_core_backward(p, p, p, p, None, p, p, p, 0.0, 1, 16, 4, 8, 1e9, p, p, p, p, None)
    assert rc == L.GTK_ERR_INVALID_ARG and b"dO_scale" in lib.gtk_last_error_string()
    assert lib.gtk_attn_core_packed_bytes(2, 10, 4, 8) == 2 * 10 * 4 * 10 * 16 * 2  # head_dim 8 pads to 16
    assert lib.gtk_attn_core_packed_bytes(1, 10, 4, 65) == 0
    assert lib.gtk_attn_core_bias_bytes(2, 10, 4) == 2 * 4 * 10 * 16 * 2  # N = 10 pads to 16
    rc = lib.gtk_attn_core_pack(p, 1, 16, 4, 65, 1.0, p, None)
    assert rc == L.GTK_ERR_INVALID_ARG
    rc = lib.gtk_attn_core_pack(p, 1, 16, 4, 8, 1.0, ctypes.c_void_p((1 << 20) + 8), None)
    assert rc == L.GTK_ERR_ALIGNMENT
    rc = lib.gtk_mha_forward(p, p, p, None, None, None, None, 1, 1, 0, 4, 2, 8, 0.3, p, None)
    assert rc == L.GTK_ERR_INVALID_ARG
    rc = lib.gtk_mha_forward(p, p, p, p, None, None, None, 1, 1, 4, 4, 2, 8, 0.3, p, None)
    assert rc == L.GTK_ERR_INVALID_ARG and b"strides" in lib.gtk_last_error_string()
    rc = lib.gtk_linear(p, None, p, None, p, 0, 8, 8, None)
    assert rc == L.GTK_ERR_INVALID_ARG
    rc = lib.gtk_linear(p, None, p, None, p, 4, 8, 8, None)
    assert rc == L.GTK_ERR_INVALID_ARG and b"alias" in lib.gtk_last_error_string()
    rc = lib.gtk_layernorm_linear(p, p, p, p, None, ctypes.c_void_p(1 << 21), 4, 8, 8, -1.0, None)
    assert rc == L.GTK_ERR_INVALID_ARG and b"eps" in lib.gtk_last_error_string()


def test_transition_entry_points(lib):
    assert lib.gtk_transition_packed_bytes(128, 4) > 2 * 128 * 512 * 2
    assert lib.gtk_transition_workspace_bytes(2, 10, 128, 4) == 2 * 10 * 10 * 512 * 2
    assert lib.gtk_transition_workspace_bytes(1, 10, 128, 2) == 10 * 10 * 512 * 2  # tuned, hidden padded to 512
    assert lib.gtk_transition_workspace_bytes(1, 10, 64, 2) > 0     # general path
    # unsupported width, then a NULL pair tensor, then a short workspace: all before any launch
    assert lib.gtk_transition_forward(None, None, None, None, 0, None, 0, 1, 16, 1024, 4, None, None) == -2
    assert lib.gtk_transition_forward(None, None, None, None, 0, None, 0, 1, 16, 128, 4, None, None) == -1
    p = ctypes.c_void_p(1 << 20)
    rc = lib.gtk_transition_forward(p, None, p, p, 1, p, 100, 1, 16, 128, 4, None, None)
    assert rc == L.GTK_ERR_WORKSPACE and b"workspace" in lib.gtk_last_error_string()
    assert lib.gtk_transition_pack(None, 128, 4, p, 1 << 20, None) == -1


def test_pair_embed_entry_points(lib):
    assert lib.gtk_pair_embed_workspace_bytes(2, 10, 128) == 2 * 2 * 10 * 128 * 4
    assert lib.gtk_pair_embed_workspace_bytes(1, 10, 64) == 2 * 10 * 64 * 4
    assert lib.gtk_pair_embed_workspace_bytes(1, 10, 4097) == 0
    p = ctypes.c_void_p(1 << 20)
    ws = lib.gtk_pair_embed_workspace_bytes(1, 16, 128)
    # c_p beyond 4096
    assert lib.gtk_pair_embed(p, None, p, None, p, None, p, ws, 1, 16, 16, 0, 32, 4097, None) == -2
    # a row shard that runs past N
    assert lib.gtk_pair_embed(p, None, p, None, p, None, p, ws, 1, 16, 8, 12, 32, 128, None) == -1
    # workspace too small
    rc = lib.gtk_pair_embed(p, None, p, None, p, None, p, ws - 4, 1, 16, 16, 0, 32, 128, None)
    assert rc == L.GTK_ERR_WORKSPACE and b"workspace" in lib.gtk_last_error_string()
    # misaligned mask
    assert lib.gtk_pair_embed(p, ctypes.c_void_p((1 << 20) + 2), p, None, p, None, p, ws, 1, 16, 16, 0, 32, 128,
                              None) == -3


def test_return_codes_match_the_header():
    text = open(HEADER).read()
    codes = dict(re.findall(r"#define\s+(GTK_(?:OK|ERR_\w+))\s+\(?(-?\d+)\)?", text))
    assert codes, "no return codes found in the header"
    for name, value in codes.items():
        assert getattr(L, name) == int(value), name


def test_noalloc_limit_is_checked_from_the_sizes_alone(lib):
    """gtk_trimul_forward_noalloc refuses sizes past its built-in scratch before it looks at
    a pointer or a device: B * N * round_up(N, 8) <= 32768."""
    for B, N in ((2, 129), (1, 256), (3, 128)):
        rc = lib.gtk_trimul_forward_noalloc(1, None, None, None, None, 0, B, N, 128, 128, None, None)
        assert rc == L.GTK_ERR_WORKSPACE, (B, N, rc)
        assert b"32768" in lib.gtk_last_error_string()
    # at the limit the size passes; the NULL pair tensor (or the missing device) is what fails
    rc = lib.gtk_trimul_forward_noalloc(1, None, None, None, None, 0, 2, 128, 128, 128, None, None)
    assert rc in (L.GTK_ERR_INVALID_ARG, L.GTK_ERR_CUDA), rc
