"""Host side of tensor parallelism, on CPU with two gloo ranks.

The NCCL unique id that rank 0 creates (hyb_nccl_unique_id) must reach every rank
unchanged, hyb_model_set_tensor_parallel must accept each rank's (rank, size, id) on an
unloaded model and reject bad ranks/sizes, and the shard rule the engine applies at
load (tp_shard_check) must accept the BASELINE TP configurations.
"""
import ctypes
import os
import socket

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import torch.distributed as dist
    import hyperion_b200 as hb
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        obj = [hb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = obj[0]
        seen = [None] * world
        dist.all_gather_object(seen, uid)
        L = hb.lib()
        m = ctypes.c_void_p()
        hb.check(L.hyp_model_create(ctypes.byref(m)))
        buf = ctypes.create_string_buffer(uid, 128)
        ok = L.hyb_model_set_tensor_parallel(m, rank, world, buf)
        bad_rank = L.hyb_model_set_tensor_parallel(m, world, world, buf)
        bad_size = L.hyb_model_set_tensor_parallel(m, 0, 9, buf)
        null_id = L.hyb_model_set_tensor_parallel(m, rank, world, None)
        L.hyp_model_free(ctypes.byref(m))
        results[rank] = (len(uid), all(x == uid for x in seen), ok, bad_rank, bad_size, null_id)
    finally:
        dist.destroy_process_group()


def test_tp_unique_id_and_rank_setup_two_gloo_ranks(built_lib):
    import torch.multiprocessing as mp
    import hyperion_b200 as hb
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(2, _free_port(), results), nprocs=2, join=True, start_method="spawn")
    for rank in range(2):
        n, same, ok, bad_rank, bad_size, null_id = results[rank]
        assert n == 128 and same
        assert ok == hb.OK
        assert bad_rank == hb.INVALID_ARGUMENT and bad_size == hb.INVALID_ARGUMENT
        assert null_id == hb.INVALID_ARGUMENT


def test_tp_shard_rule():
    import hyperion_b200 as hb
    from hyperion_b200.synth import config0, config3, config4
    for tp in (1, 2, 4, 8):
        assert hb.tp_shard_check(config4(), tp) is None  # 27B shape: the BASELINE TP config
    assert hb.tp_shard_check(config3(), 8) is None
    assert hb.tp_shard_check(config0(), 2) is None
    assert "split evenly" in hb.tp_shard_check(config0(), 8)
    assert hb.tp_shard_check(config4(), 16) is not None
