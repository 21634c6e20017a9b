"""Spawn `world` CPU ranks (gloo, 127.0.0.1 rendezvous) running `fn(rank, world, *args)`."""
import os
import socket

import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn, args):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="")
    import torch
    torch.set_num_threads(2)
    fn(rank, world, *args)


def spawn(fn, world, *args, timeout=300):
    ctx = mp.start_processes(_entry, args=(world, free_port(), fn, args), nprocs=world, join=False, start_method="spawn")
    import time
    t0 = time.time()
    while not ctx.join(timeout=5):
        if time.time() - t0 > timeout:
            for p in ctx.processes:
                p.terminate()
            raise TimeoutError(f"spawned ranks did not finish in {timeout}s")
