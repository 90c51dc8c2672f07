"""Ulysses sequence-parallel bookkeeping on CPU: shard geometry from the library's own
ernie_cuda_sp_layout, and the two all-to-alls and the latent gather replayed with world_size-2 gloo
point-to-point transfers using exactly the block offsets the CUDA session uses (per (peer, head) blocks of
S x 128 into [heads/P][F][128]; [P][S][heads/P x 128] back; [P][128][S] latent slices). No GPU.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import ernie_cuda as ec

HEADS, DIM = 32, 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("tokens,image", [(8256, 8192), (216, 192), (88, 48), (16, 8), (6176, 4128)])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_layout_covers_every_token_once(tokens, image, world):
    covered_img, covered_all, text_slots = [], [], []
    for r in range(world):
        S, F, img, real, tb = ec.sp_layout(tokens, image, world, r)
        assert S % 16 == 0 and F % 128 == 0 and F >= world * S >= tokens
        assert 0 <= img <= real <= S
        begin = r * S
        covered_img += list(range(begin, begin + img))
        covered_all += list(range(begin, begin + real))
        text_slots += list(range(tb, tb + real - img))
        if img < real:  # a shard's text rows continue the global sequence right after its image rows
            assert begin + img - image == tb
    assert covered_img == list(range(image))
    assert covered_all == list(range(tokens))
    assert text_slots == list(range(tokens - image))


def global_qkv(tokens):
    """Deterministic per-(tensor, head, token, dim) values, so any misplaced block shows up."""
    t = np.arange(3)[:, None, None, None]
    h = np.arange(HEADS)[None, :, None, None]
    n = np.arange(tokens)[None, None, :, None]
    d = np.arange(DIM)[None, None, None, :]
    return (((t * HEADS + h) * 16384 + n) * 4 + d % 4).astype(np.float64)


def _worker(rank, world, port, tokens, image, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        S, F, img, real, _ = ec.sp_layout(tokens, image, world, rank)
        hl = HEADS // world
        g = global_qkv(tokens)
        # send buffers: this rank's rows of all 32 heads, [32][S][128], rows past `real` zero
        send = np.zeros((3, HEADS, S, DIM))
        send[:, :, :real] = g[:, :, rank * S: rank * S + real]
        recv = np.zeros((3, hl, F, DIM))
        ops = []
        recv_views = []
        for t in range(3):
            for peer in range(world):
                for h in range(hl):
                    block = torch.from_numpy(np.ascontiguousarray(send[t, peer * hl + h]))
                    buf = torch.empty_like(block)
                    recv_views.append((t, h, peer, buf))
                    if peer == rank:
                        buf.copy_(block)
                    else:
                        ops.append(dist.P2POp(dist.isend, block, peer))
                        ops.append(dist.P2POp(dist.irecv, buf, peer))
        for req in dist.batch_isend_irecv(ops) if ops else []:
            req.wait()
        for t, h, peer, buf in recv_views:
            recv[t, h, peer * S: (peer + 1) * S] = buf.numpy()
        # the gathered sequence of this rank's heads must be the global one, zero padded
        expect = np.zeros((3, hl, F, DIM))
        expect[:, :, :tokens] = g[:, rank * hl: (rank + 1) * hl]
        qkv_ok = bool(np.array_equal(recv, expect))
        # attention rows of every token for this rank's heads go back to the owning rank
        o_full = np.zeros((F, hl * DIM))
        o_full[:tokens] = recv[0, :, :tokens].transpose(1, 0, 2).reshape(tokens, hl * DIM)
        o_recv = np.zeros((world, S, hl * DIM))
        ops = []
        bufs = []
        for peer in range(world):
            block = torch.from_numpy(np.ascontiguousarray(o_full[peer * S: (peer + 1) * S]))
            buf = torch.empty_like(block)
            bufs.append((peer, buf))
            if peer == rank:
                buf.copy_(block)
            else:
                ops.append(dist.P2POp(dist.isend, block, peer))
                ops.append(dist.P2POp(dist.irecv, buf, peer))
        for req in dist.batch_isend_irecv(ops) if ops else []:
            req.wait()
        for peer, buf in bufs:
            o_recv[peer] = buf.numpy()
        # gather_heads: [P][S][hl*128] -> [S][4096]
        a = o_recv.transpose(1, 0, 2).reshape(S, HEADS * DIM)
        mine = g[0, :, rank * S: rank * S + real].transpose(1, 0, 2).reshape(real, HEADS * DIM)
        o_ok = bool(np.array_equal(a[:real], mine))
        # latent: [128][S] slices gathered into [P][128][S], reassembled into [128][image]
        lat = np.arange(128 * image, dtype=np.float64).reshape(128, image)
        slice_ = np.zeros((128, S))
        slice_[:, :img] = lat[:, rank * S: rank * S + img]
        gathered = [torch.zeros(128, S, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(slice_))
        out = np.zeros_like(lat)
        for p in range(world):
            img_p = max(0, min(S, image - p * S))
            out[:, p * S: p * S + img_p] = gathered[p].numpy()[:, :img_p]
        results[rank] = (qkv_ok, o_ok, bool(np.array_equal(out, lat)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens,image", [(216, 192), (88, 48), (16, 8)])
def test_two_rank_exchange_replay(tokens, image):
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(2, port, tokens, image, results), nprocs=2, join=True, start_method="spawn")
    assert dict(results) == {0: (True, True, True), 1: (True, True, True)}
