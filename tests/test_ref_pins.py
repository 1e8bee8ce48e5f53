"""Pins against the reference's own compiled code (CPU; needs the reference tree,
whose MLX-free sources oracle/build_oracle.py compiles into oracle/_ref/).

* ring / global KV index arithmetic: native/hyperion_mlx/src/kv.cc via ref_shim;
  compared with the oracle's rings and the slot rule the CUDA kernels use;
* geometry validation: native/hyperion_mlx/src/geometry.cc compared with this
  library's hyp_model_load verdicts (validation runs before any CUDA call);
* the tiny fixture's tensor layout (names, dtypes, shapes) compared with the
  synthetic checkpoints this repository writes.
"""
import ctypes
import os

import numpy as np
import pytest

from oracle.build_oracle import REF, build_ref, reference_present

pytestmark = pytest.mark.skipif(not reference_present(), reason="reference tree not mounted")


@pytest.fixture(scope="module")
def ref_index():
    built = build_ref()
    L = ctypes.CDLL(built["index"])
    L.ref_ring_slots.restype = ctypes.c_uint32
    L.ref_ring_slots.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_uint32]
    L.ref_ring_capacity.restype = ctypes.c_uint32
    L.ref_ring_capacity.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
    L.ref_global_capacities.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    L.ref_geometry_check.restype = ctypes.c_int
    L.ref_geometry_check.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    return L


@pytest.mark.parametrize("window,commits", [(1024, [2048, 1, 1, 1]), (128, [32, 1, 200, 7]),
                                            (8, [3, 9, 1, 20]), (1024, [2048, 2048, 513])])
def test_ring_slots_match_reference(ref_index, window, commits):
    from oracle.gemma_oracle import LocalRing
    c = np.asarray(commits, dtype=np.uint32)
    n_pos = int(c.sum()) + 5
    slots = np.zeros(n_pos, dtype=np.uint32)
    committed = ref_index.ref_ring_slots(window, 8, c.ctypes.data, len(c), slots.ctypes.data, n_pos)
    cap = ref_index.ref_ring_capacity(window, 8)
    assert cap == window + 8
    assert committed == c.sum()
    ours = np.arange(n_pos) % (window + 8)  # the kernels' slot rule
    assert np.array_equal(slots, ours)
    ring = LocalRing(window, 1, 64)
    assert all(ring.slot_for(p) == slots[p] for p in range(n_pos))


@pytest.mark.parametrize("appends", [[256, 1, 1024], [1, 255, 1, 0, 300], [4096, 1, 1, 1], [20, 1, 1]])
def test_global_capacity_steps_match_reference(ref_index, appends):
    from oracle.gemma_oracle import GlobalCache
    a = np.asarray(appends, dtype=np.uint32)
    caps = np.zeros(len(a), dtype=np.uint32)
    ref_index.ref_global_capacities(256, a.ctypes.data, len(a), caps.ctypes.data)
    g = GlobalCache(1, 64)
    for i, n in enumerate(appends):
        if n:
            g.append(np.zeros((n, 1, 64), np.uint16), np.zeros((n, 1, 64), np.uint16))
        assert g.capacity() == caps[i]


def _geometries():
    from hyperion_b200.synth import config0, config3, tiny_fixture_geometry
    import hyperion_b200 as hb
    cases = []
    for geo in (config0(), config3(), tiny_fixture_geometry()):
        cases.append(("valid", hb.geometry_params(geo)))
    def mut(fn, label):
        p = hb.geometry_params(config0())
        fn(p)
        cases.append((label, p))
    mut(lambda p: setattr(p, "num_hidden_layers", 0), "zero layers")
    mut(lambda p: setattr(p, "sliding_window", 0), "zero window")
    mut(lambda p: setattr(p, "vocab_size", 0), "zero vocab")
    mut(lambda p: setattr(p, "tie_word_embeddings", 0), "untied")
    mut(lambda p: setattr(p, "num_kv_heads_local", 0), "zero kv heads")
    mut(lambda p: setattr(p.rope_global, "proportional", 0), "global rope not proportional")
    mut(lambda p: setattr(p.rope_local, "has_partial_rotary_factor", 1), "local partial")
    mut(lambda p: setattr(p.rope_local, "theta", -1.0), "negative theta")
    mut(lambda p: setattr(p, "model_type", 7), "bad model type")
    mut(lambda p: setattr(p, "num_kv_shared_layers", 99), "kv shared > layers")
    def last_sliding(p):
        arr = (ctypes.c_int * 2)(1, 0)
        p._layer_arr = arr
        p.layer_types = ctypes.cast(arr, ctypes.POINTER(ctypes.c_int))
    mut(last_sliding, "last layer sliding")
    def bad_kind(p):
        arr = (ctypes.c_int * 2)(0, 5)
        p._layer_arr = arr
        p.layer_types = ctypes.cast(arr, ctypes.POINTER(ctypes.c_int))
    mut(bad_kind, "bad layer kind")
    def null_types(p):
        p.layer_types = ctypes.cast(None, ctypes.POINTER(ctypes.c_int))
    mut(null_types, "null layer types")
    return cases


def test_geometry_validation_matches_reference(ref_index, built_lib):
    import hyperion_b200 as hb
    for label, p in _geometries():
        msg = ctypes.create_string_buffer(512)
        verdict = ref_index.ref_geometry_check(ctypes.byref(p), msg, 512)
        m = ctypes.c_void_p()
        hb.check(built_lib.hyp_model_create(ctypes.byref(m)))
        st = built_lib.hyp_model_load(m, ctypes.byref(p), b"/nonexistent/weights/dir")
        err = hb.last_error()
        built_lib.hyp_model_free(ctypes.byref(m))
        if verdict == 0:
            assert st == hb.NOT_FOUND, (label, st, err)
        else:
            assert st == hb.INVALID_ARGUMENT, (label, st, err)
            assert err == msg.value.decode(), (label, err, msg.value)


def test_tiny_fixture_layout_matches_synthetic_writer(tmp_path):
    from hyperion_b200.safetensors_io import read_checkpoint_dir
    from hyperion_b200.synth import tiny_fixture_geometry, write_checkpoint
    ref = read_checkpoint_dir(os.path.join(REF, "crates/hyperion-model/fixtures/gemma4-unified-tiny"))
    ours = write_checkpoint(tiny_fixture_geometry(), str(tmp_path), seed=0)
    assert set(ref) == set(ours)
    for name in ref:
        assert ref[name].dtype == ours[name].dtype, name
        assert tuple(ref[name].shape) == tuple(ours[name].shape), name
    # the reference fixture is itself readable by the oracle (global layer 5 has no v_proj)
    assert "language_model.model.layers.5.self_attn.v_proj.weight" not in ref
