"""One rank of the sequence-parallel parity run (started by test_gpu_sp.py, one process per GPU).

Every rank builds the same synthetic model and a Ulysses session member; the members swap their
64-byte memory handles through files in ERNIE_SP_DIR (each written, then renamed) and denoise the same
seeded latent. Rank 0 then denoises the same request with a single-GPU session on its own device and
writes both results to ERNIE_SP_DIR/sp.npz.
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
    folder = os.environ["ERNIE_SP_DIR"]

    def exchange(handle):
        mine = os.path.join(folder, f"handle{rank}")
        with open(mine + ".tmp", "wb") as f:
            f.write(handle)
        os.replace(mine + ".tmp", mine)
        handles = []
        deadline = time.time() + 120
        for r in range(world):
            path = os.path.join(folder, f"handle{r}")
            while not os.path.exists(path):
                if time.time() > deadline:
                    raise SystemExit(f"rank {r} never published its handle")
                time.sleep(0.05)
            with open(path, "rb") as f:
                handles.append(f.read())
        return handles

    ctx = ec.Context(rank)
    model = ec.Model(ctx, blocks)
    model.synthesize(11)
    rng = np.random.default_rng(5)
    latent = rng.standard_normal((128, h, w), dtype=np.float32)
    text_in = rng.standard_normal((text, 3072), dtype=np.float32)
    cos, sin, mask = ec.dit_constants(w, h, valid, text)
    s = ec.Session(model, w, h, text, valid, ec.BF16, sp=(rank, world, exchange))
    s.set_conditioning(text_in, cos, sin, mask)
    got = s.denoise(latent, steps, 0, end)
    again = s.denoise(latent, steps, 0, end)
    s.close()
    if rank == 0:
        single = ec.Session(model, w, h, text, valid, ec.BF16)
        single.set_conditioning(text_in, cos, sin, mask)
        ref = single.denoise(latent, steps, 0, end)
        single.close()
        np.savez(os.path.join(folder, "sp.npz"), sp=got, sp_again=again, single=ref)
    model.close()
    ctx.close()


if __name__ == "__main__":
    main()
