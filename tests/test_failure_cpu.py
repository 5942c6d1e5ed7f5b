"""Failure detection on CPU ranks (gloo): heartbeats on the c10d store, host-side
fault injection, and a trainer whose peer leaves between steps.  No GPU involved."""
import os
import socket
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_parse_fault_spec():
    from tinytron_b200.utils.watchdog import fault_active, parse_fault_spec

    spec = "exit@1:3, hang_heartbeat@2,skip_signal@0"
    assert parse_fault_spec(spec) == [("exit", 1, 3), ("hang_heartbeat", 2, None), ("skip_signal", 0, None)]
    assert fault_active("exit", 1, 3, spec) and not fault_active("exit", 1, 2, spec)
    assert fault_active("hang_heartbeat", 2, None, spec) and not fault_active("hang_heartbeat", 1, None, spec)
    with pytest.raises(ValueError):
        parse_fault_spec("exit")


def _hb_worker(rank, world, port, scenario, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if scenario == "silent" and rank == world - 1:
        os.environ["TT_FAULT_INJECT"] = f"hang_heartbeat@{rank}"
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from tinytron_b200.utils.watchdog import Heartbeat, PeerFailure

    hb = Heartbeat(rank, world, interval=0.1, timeout=1.0)
    result = None
    victim = world - 1
    if rank == victim:
        if scenario == "exit":
            time.sleep(0.5)
            hb.close(exit_code=1)
        else:
            time.sleep(4.0)
        result = "victim"
    else:
        t0 = time.time()
        while time.time() - t0 < 8.0:
            try:
                hb.check()
            except PeerFailure as exc:
                result = exc.ranks
                break
            time.sleep(0.1)
    q.put((rank, result))
    time.sleep(1.0)  # keep the store (rank 0) alive while the others read it
    if rank != victim or scenario != "exit":
        hb.close(0)


@pytest.mark.parametrize("scenario", ["silent", "exit"])
def test_heartbeat_detects_failed_peer(scenario):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 3, _port()
    procs = [ctx.Process(target=_hb_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[0] == [world - 1] and res[1] == [world - 1], res


def _trainer_worker(rank, world, port, log_dir, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), TT_FAULT_INJECT="exit@1:2", TT_HEARTBEAT_TIMEOUT_S="3",
                      TT_PG_TIMEOUT_S="15")
    from tinytron_b200.training import build_config, parse_args
    from tinytron_b200.training.trainer import Trainer

    argv = ["--use_mock_data", "--mock_data_num_samples", "64", "--log_dir", log_dir, "--total_batch_size", "512",
            "--batch_size", "2", "--seq_len", "32", "--max_steps", "6", "--warmup_steps", "1", "--debug",
            "--backend", "gloo", "--num_layer", "1", "--hidden_size", "64", "--num_attention_heads", "4",
            "--num_key_value_heads", "2", "--intermediate_size", "128", "--vocab_size", "256", "--block_size", "64"]
    t0 = time.time()
    try:
        Trainer(build_config(parse_args(argv))).train()
        outcome = "finished"
    except Exception as exc:
        outcome = type(exc).__name__
    q.put((rank, outcome, time.time() - t0))


def test_trainer_peer_exit_is_detected(tmp_path):
    """Rank 1 leaves between steps (injected); rank 0 must stop with an error (the
    heartbeat's PeerFailure, or its next collective timing out), never hang."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_trainer_worker, args=(r, 2, port, str(tmp_path), q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, outcome, dt = q.get(timeout=180)
        res[r] = (outcome, dt)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1][0] == "InjectedFault", res
    assert res[0][0] in ("PeerFailure", "RuntimeError", "DistBackendError"), res
