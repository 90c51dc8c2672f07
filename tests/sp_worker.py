"""One rank of the sequence-parallel parity run (started by test_gpu_sp.py, one process per GPU).

Rank 0 makes the NCCL id and publishes it in the file ERNIE_SP_ID_FILE (written, then renamed); every
rank builds the same synthetic model, joins a Ulysses session with that id, and denoises the same seeded
latent. Rank 0 then denoises the same request with a single-GPU session on its own device and writes
both results to ERNIE_SP_OUT (.npz). All ranks load the same libnccl.so.2 (none imports torch).
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "ernie-image-ncnn-vulkan_b200"))

import ernie_cuda as ec  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    w, h, text, valid, blocks, steps, end = (int(v) for v in os.environ["ERNIE_SP_CASE"].split(","))
    id_file = os.environ["ERNIE_SP_ID_FILE"]
    if rank == 0:
        with open(id_file + ".tmp", "wb") as f:
            f.write(ec.nccl_unique_id())
        os.replace(id_file + ".tmp", id_file)
    deadline = time.time() + 120
    while not os.path.exists(id_file):
        if time.time() > deadline:
            raise SystemExit("rank 0 never published the NCCL id")
        time.sleep(0.05)
    with open(id_file, "rb") as f:
        nccl_id = f.read()
    ctx = ec.Context(rank)
    model = ec.Model(ctx, blocks)
    model.synthesize(11)
    rng = np.random.default_rng(5)
    latent = rng.standard_normal((128, h, w), dtype=np.float32)
    text_in = rng.standard_normal((text, 3072), dtype=np.float32)
    cos, sin, mask = ec.dit_constants(w, h, valid, text)
    s = ec.Session(model, w, h, text, valid, ec.BF16, sp=(nccl_id, rank, world))
    s.set_conditioning(text_in, cos, sin, mask)
    got = s.denoise(latent, steps, 0, end)
    again = s.denoise(latent, steps, 0, end)
    s.close()
    if rank == 0:
        single = ec.Session(model, w, h, text, valid, ec.BF16)
        single.set_conditioning(text_in, cos, sin, mask)
        ref = single.denoise(latent, steps, 0, end)
        single.close()
        np.savez(os.environ["ERNIE_SP_OUT"], sp=got, sp_again=again, single=ref)
    model.close()
    ctx.close()


if __name__ == "__main__":
    main()
