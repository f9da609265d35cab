"""Multi-process host logic of the sharded paths, on CPU with the gloo backend (world 2).

What runs on GPUs with NCCL is the same code: row/column sharding and the single
all_gather_into_tensor of column-sharded outputs.  The local int8 GEMM is stood in for by
the oracle here (no GPU), which also makes the reassembled result checkable bit for bit.
"""

import datetime
import multiprocessing as mp
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch

from conftest import PKG, ROOT


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=30):
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    # The rendezvous gets its own generous limit (spawned ranks may take a while to import
    # torch on a loaded machine); timeout_s bounds the collectives only.
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=120))
    dist.init_process_group(
        "gloo", store=store, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s)
    )
    return dist


def _worker_gather(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        from llm_kernels.sharding import gather_columns, gather_rows, shard_range, shard_rows

        g = torch.Generator().manual_seed(5)
        full = torch.randn(11, 13, generator=g)
        rows = gather_rows(shard_rows(full, rank, world).clone(), 11)
        assert torch.equal(rows, full)
        s, e = shard_range(13, rank, world)
        cols = gather_columns(full[:, s:e].contiguous(), 13)
        assert torch.equal(cols, full)
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _worker_tp_gemm(rank, world, port, q):
    """Column-sharded int8 linear: quantise x (replicated), local GEMM on this rank's N/g
    weight rows, gather.  The gathered [M, N] must equal the unsharded result exactly."""
    try:
        dist = _init(rank, world, port)
        import oracle
        from llm_kernels.sharding import gather_columns, shard_columns

        g = torch.Generator().manual_seed(9)
        x = torch.randn(24, 64, generator=g).to(torch.float16)
        w = torch.randn(50, 64, generator=g).to(torch.float16)
        xq, sx = oracle.quantize_symmetric(x)
        wq, sw = oracle.quantize_symmetric(w)
        wq_t, sw_t = torch.from_numpy(wq), torch.from_numpy(sw)
        wq_r = shard_columns(wq_t, rank, world)
        sw_r = shard_columns(sw_t[:, None], rank, world)[:, 0]
        y_r = oracle.int8_gemm_dequant(xq, wq_r.numpy(), sx, sw_r.numpy(), "nk")
        y = gather_columns(torch.from_numpy(y_r), 50)
        ref = oracle.int8_gemm_dequant(xq, wq, sx, sw, "nk")
        assert np.array_equal(y.numpy().view(np.uint16), ref.view(np.uint16))
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _worker_rank_fails(rank, world, port, q):
    """Rank 1 fails between steps (raises before the collective); rank 0 must get an error
    from its next collective within the process-group timeout instead of hanging."""
    try:
        dist = _init(rank, world, port, timeout_s=5)
        from llm_kernels.sharding import gather_rows

        if rank == 1:
            raise RuntimeError("planted failure on rank 1")
        try:
            gather_rows(torch.ones(2, 3), 4)
            q.put((rank, "no error"))
        except Exception as e:  # expected: timeout or closed connection
            q.put((rank, "error:" + type(e).__name__))
    except RuntimeError as e:
        q.put((rank, "raised:" + str(e)))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _run(worker, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            r, msg = q.get(timeout=timeout)
            out[r] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return out


def test_shard_range_partitions_exactly():
    from llm_kernels.sharding import shard_range

    for n in (0, 1, 7, 64, 1000):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_gather_rows_and_columns_world2():
    out = _run(_worker_gather)
    assert out == {0: "ok", 1: "ok"}, out


def test_column_sharded_int8_linear_matches_unsharded_world2():
    out = _run(_worker_tp_gemm)
    assert out == {0: "ok", 1: "ok"}, out


def test_failed_rank_surfaces_as_error_not_hang():
    out = _run(_worker_rank_fails, timeout=90)
    assert out[1].startswith("raised:planted failure")
    assert out[0].startswith("error:"), out[0]


@pytest.mark.gpu
def test_column_sharded_path_on_gpu_world1_nccl():
    """The CUDA path of the column-sharded linear with an NCCL group of one rank."""
    import torch.distributed as dist

    import llm_kernels
    import oracle
    from llm_kernels.sharding import column_sharded_int8_linear

    if not dist.is_initialized():
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(_free_port())
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(3)
        x = torch.randn(40, 256, generator=g).to(torch.float16).cuda()
        layer = llm_kernels.Int8Linear(256, 96)
        layer.quantize_weights(torch.randn(96, 256, generator=g).to(torch.float16).cuda())
        y = column_sharded_int8_linear(x, layer.w_q, layer.scale_w, 96)
        assert torch.equal(y, layer(x))
        xq, sx = oracle.quantize_symmetric(x.cpu())
        ref = oracle.int8_gemm_dequant(xq, layer.w_q.cpu().numpy(), sx, layer.scale_w.cpu().numpy(), "nk")
        assert np.array_equal(y.cpu().numpy().view(np.uint16), ref.view(np.uint16))
    finally:
        dist.destroy_process_group()


def _worker_fused_gather_gpu(rank, world, port, q):
    """One rank of the column-sharded int8 linear on GPU `rank`: the fused-epilogue gather
    (peer stores over NVLink) and the NCCL all-gather path must both equal the unsharded
    Int8Linear bit for bit, on two calls in a row."""
    try:
        for p in (ROOT, PKG):
            if p not in sys.path:
                sys.path.insert(0, p)
        torch.cuda.set_device(rank)
        import torch.distributed as dist

        store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=120))
        dist.init_process_group("nccl", store=store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device(f"cuda:{rank}"))
        import llm_kernels
        from llm_kernels.sharding import (MulticastBuffers, PeerBuffers, column_sharded_int8_linear,
                                          column_sharded_int8_linear_fused, column_sharded_int8_linear_multicast)
        from llm_kernels.sharding import shard_columns

        results = []
        multicast_ran, no_mc = False, ""
        for M, K, N in ((1000, 512, 768), (4096, 4096, 4096)):
            g = torch.Generator().manual_seed(M + N)
            x = torch.randn(M, K, generator=g).to(torch.float16).cuda()
            w = torch.randn(N, K, generator=g).to(torch.float16).cuda()
            layer = llm_kernels.Int8Linear(K, N).cuda()
            layer.quantize_weights(w)
            ref = layer(x)
            wq_r = shard_columns(layer.w_q, rank, world)
            sw_r = shard_columns(layer.scale_w[:, None], rank, world)[:, 0].contiguous()
            buf = PeerBuffers((M, N))
            for _ in range(2):
                y = column_sharded_int8_linear_fused(x, wq_r, sw_r, buf)
                results.append(bool(torch.equal(y, ref)))
            results.append(bool(torch.equal(column_sharded_int8_linear(x, wq_r, sw_r, N), ref)))
            # A second set of buffers while the first is open: on a peer both usually sit in one
            # caching-allocator segment, i.e. arrive with the same IPC handle.  Closing the first
            # must leave the second mapped.
            buf2 = PeerBuffers((M, N))
            y2 = column_sharded_int8_linear_fused(x, wq_r, sw_r, buf2)
            results.append(bool(torch.equal(y2, ref)))
            buf.close()
            y2 = column_sharded_int8_linear_fused(x, wq_r, sw_r, buf2)
            results.append(bool(torch.equal(y2, ref)))
            buf2.close()
            # The NVSwitch-multicast gather (multimem stores), where the GPUs support it.
            try:
                mbuf = MulticastBuffers((M, N))
            except Exception as e:  # noqa: BLE001  (no NVLS / no symmetric memory here)
                mbuf, no_mc = None, str(e)[:80]
            if mbuf is not None:
                for _ in range(2):
                    y3 = column_sharded_int8_linear_multicast(x, wq_r, sw_r, mbuf)
                    torch.cuda.synchronize()
                    results.append(bool(torch.equal(y3, ref)))
                mbuf.close()
                multicast_ran = True
        dist.destroy_process_group()
        q.put((rank, ("ok" if multicast_ran else f"ok (no multicast: {no_mc})") if all(results) else f"mismatch {results}"))
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_column_sharded_fused_gather_on_all_gpus():
    """Every GPU of the box (2 to 8) as one rank: per-rank column blocks of 384 / 192 / 96
    (one-CTA kernel) and 2048 / 1024 / 512 columns (CTA-pair kernel at 2 ranks)."""
    world = min(torch.cuda.device_count(), 8)
    out = _run(_worker_fused_gather_gpu, world=world, timeout=300)
    assert all(v.startswith("ok") for v in out.values()) and len(out) == world, out
    print("fused gather on", world, "GPUs:", sorted(set(out.values())))
