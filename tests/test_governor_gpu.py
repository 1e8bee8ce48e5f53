"""Governor admission, staged KV growth and memory telemetry through the 14-function ABI.

Reference semantics (paths inside jscott3201/hyperion):
  * predictive admission runs before any work and rejects with OOM_GOVERNOR, the step
    result carrying HYP_GOVERNOR_HARD_REJECT (model.cc:665-683, governor.h:148-186);
  * a call whose plan crosses a global-cache capacity bucket runs against a staged
    state that is published only on success (KvGrowthTransaction, kv_cache.h:220-261,
    kv_cache.cc:68-128), so a failure leaves the live state and its cursor usable;
  * a call without growth executes directly and a failure after the first forward
    consumes the state (model.cc:79-105).
The failure is injected on the host (hyb_test_arm_post_append_fault); no GPU fault is
involved. The budget is the engine's memory ceiling (hyb_model_set_memory_budget).
"""
import ctypes

import numpy as np
import pytest

import hyperion_b200 as hb
from hyperion_b200.synth import config0
from tests.conftest import has_gpu

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_gpu(), reason="no CUDA device")]

HARD_REJECT = 2
GLOBAL_ROW = 2 * 64 * 2 * 2  # cfg0 global layer: 2 KV heads x hd 64, K and V, bf16


def _prompt(n, seed=1):
    return np.random.default_rng(seed).integers(0, 1024, n).tolist()


def _decode(eng, kv, n):
    L = hb.lib()
    st = L.hyp_decode_block(eng.handle, kv.handle, n, eng._result)
    return st, eng.fields()


def test_admission_rejects_growth_above_budget_before_any_work(built_lib):
    eng = hb.Engine(config0(), synthetic_seed=4)
    kv, twin = eng.new_kv(), eng.new_kv()
    kv.prefill(_prompt(249))
    twin.prefill(_prompt(249))
    f, _ = kv.decode(1)  # the first decode step sizes the decode workspace
    twin.decode(1)
    assert f.global_kv_bytes == 256 * GLOBAL_ROW and f.peak_mlx_bytes >= f.active_mlx_bytes
    before = kv.cursor()
    assert before[0] == 250
    eng.set_memory_budget(f.active_mlx_bytes + 1024)  # no room for a staged 512-token global cache
    st, fr = _decode(eng, kv, 10)  # 250 -> 260 crosses the 256-token bucket
    assert st == hb.OOM_GOVERNOR, hb.STATUS_NAMES[st]
    assert "memory budget" in hb.last_error()
    assert fr.governor_state == HARD_REJECT and fr.token_id == 0
    assert kv.cursor() == before  # rejected before any work
    assert fr.global_kv_bytes == 256 * GLOBAL_ROW
    # a block that stays inside the bucket needs no new device memory and is admitted
    st, fr = _decode(eng, kv, 6)
    assert st == hb.OK and fr.governor_state == 0 and kv.cursor()[0] == 256
    # lift the ceiling: the state decodes on exactly like a twin that was never rejected
    eng.set_memory_budget(0)
    _, ft = _decode(eng, twin, 6)
    assert ft.token_id == fr.token_id
    for _ in range(8):
        a, _ = kv.decode(1)
        b, _ = twin.decode(1)
        assert a.token_id == b.token_id
    assert kv.cursor() == twin.cursor()


@pytest.mark.parametrize("n_tokens", [4, 12])
def test_failed_growth_call_rolls_back(built_lib, n_tokens):
    """n_tokens 4 writes only ring slack; 12 exceeds it and takes the ring backup path."""
    eng = hb.Engine(config0(), synthetic_seed=5)
    kv, twin = eng.new_kv(), eng.new_kv()
    p = _prompt(254, seed=3)  # 254 + 4 and 254 + 12 both cross the 256-token bucket
    kv.prefill(p)
    twin.prefill(p)
    before = kv.cursor()
    hb.check(hb.lib().hyb_test_arm_post_append_fault())
    st, _ = _decode(eng, kv, n_tokens)  # crosses 256: staged, then the injected failure
    assert st == hb.INTERNAL and "injected" in hb.last_error()
    assert kv.cursor() == before
    # not poisoned: it decodes the same block as the twin that never failed
    st, fa = _decode(eng, kv, n_tokens)
    assert st == hb.OK, hb.last_error()
    _, fb = _decode(eng, twin, n_tokens)
    assert fa.token_id == fb.token_id and kv.cursor() == twin.cursor()
    assert fa.global_kv_bytes == 512 * GLOBAL_ROW
    for _ in range(6):
        a, la = kv.decode(1, logits=True)
        b, lb = twin.decode(1, logits=True)
        assert a.token_id == b.token_id and np.array_equal(la, lb)


def test_failed_prefill_leaves_state_fresh(built_lib):
    eng = hb.Engine(config0(), synthetic_seed=6)
    kv, twin = eng.new_kv(), eng.new_kv()
    hb.check(hb.lib().hyb_test_arm_post_append_fault())
    arr = (ctypes.c_uint32 * 40)(*_prompt(40))
    ts = hb.HypTokenStream(ctypes.cast(arr, ctypes.POINTER(ctypes.c_uint32)), 40, 1)
    st = hb.lib().hyp_prefill_chunk(eng.handle, kv.handle, ctypes.byref(ts), eng._result)
    assert st == hb.INTERNAL and "injected" in hb.last_error()
    assert kv.cursor() == (0, 0)
    f, la = kv.prefill(_prompt(40), logits=True)  # the state is still fresh and usable
    g, lb = twin.prefill(_prompt(40), logits=True)
    assert f.token_id == g.token_id and np.array_equal(la, lb)


def test_failure_without_growth_consumes_the_state(built_lib):
    eng = hb.Engine(config0(), synthetic_seed=7)
    kv = eng.new_kv()
    kv.prefill(_prompt(20))
    hb.check(hb.lib().hyb_test_arm_post_append_fault())
    assert _decode(eng, kv, 1)[0] == hb.INTERNAL
    assert _decode(eng, kv, 1)[0] == hb.INTERNAL and "free and recreate" in hb.last_error()


def test_peak_bytes_cover_the_staged_growth(built_lib):
    """The growth step holds the old and the new global buffers at once: the call's peak
    exceeds the bytes still allocated after it published by the freed old buffers."""
    eng = hb.Engine(config0(), synthetic_seed=8)
    kv = eng.new_kv()
    kv.prefill(_prompt(255))
    st, f = _decode(eng, kv, 2)  # 255 -> 257: 256 -> 512 rows
    assert st == hb.OK
    assert f.global_kv_bytes == 512 * GLOBAL_ROW
    assert f.peak_mlx_bytes >= f.active_mlx_bytes + 256 * GLOBAL_ROW
    st, f2 = _decode(eng, kv, 1)  # no growth: the peak is the live allocation
    assert f2.peak_mlx_bytes == f2.active_mlx_bytes
