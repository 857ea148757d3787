"""Helpers to run a function on N local ranks (gloo on CPU or nccl on GPUs).

Ranks rendezvous through a file store in a fresh temporary directory, so
concurrent or back-to-back runs never race for a TCP port."""
import os
import shutil
import socket
import tempfile
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, backend, fn, args, errq, final_barrier=True, pg_timeout=60,
           store_path=None):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        if backend == "nccl":
            torch.cuda.set_device(rank)
        import datetime
        dist.init_process_group(backend, init_method=f"file://{store_path}", rank=rank,
                                world_size=world,
                                timeout=datetime.timedelta(seconds=pg_timeout),
                                **({"device_id": torch.device("cuda", rank)} if backend == "nccl" else {}))
        fn(rank, world, *args)
        if final_barrier:
            dist.barrier()
    except BaseException:
        errq.put((rank, traceback.format_exc()))
        raise
    finally:
        if dist.is_initialized() and final_barrier:
            dist.destroy_process_group()


def run_ranks(fn, world, *args, backend="gloo", timeout=240, final_barrier=True, pg_timeout=60,
              env=None):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()  # exported as MASTER_PORT for code that reads it; not bound
    tmp = tempfile.mkdtemp(prefix="mgfa_pg_")
    store_path = os.path.join(tmp, "store")
    saved = {k: os.environ.get(k) for k in (env or {})}
    os.environ.update(env or {})
    procs = [ctx.Process(target=_entry, args=(r, world, port, backend, fn, args, errq,
                                               final_barrier, pg_timeout, store_path))
             for r in range(world)]
    for p in procs:
        p.start()
    for k, v in saved.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    shutil.rmtree(tmp, ignore_errors=True)
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    if errors:
        raise AssertionError("rank failures:\n" + "\n".join(f"[rank {r}]\n{tb}" for r, tb in errors))
    if alive:
        raise AssertionError(f"{len(alive)} rank(s) did not finish within {timeout}s")
    bad = [p.exitcode for p in procs if p.exitcode != 0]
    if bad:
        raise AssertionError(f"rank exit codes {bad}")
