"""Launched by tests/test_failure_cpu.py under torch.distributed.run: rank 1
exits with an error right after the rendezvous, rank 0 keeps working; the
launcher must notice and stop the job."""
import os
import sys
import time

import torch.distributed as dist

dist.init_process_group("gloo")
rank = dist.get_rank()
if rank == 1:
    sys.stdout.flush()
    os._exit(7)
t0 = time.time()
while time.time() - t0 < 120:
    time.sleep(0.2)
print("rank 0 was never stopped", flush=True)
