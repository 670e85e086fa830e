"""CPU restatement of the reference's tensor-parallel decode over its gRPC all-reduce.

TEST / BASELINE INFRASTRUCTURE ONLY.  ``bench.py``'s reference arm times this module
on the GPU host's own cores as the stand-in for the reference's CPU path (the
reference's Python sources, and the protobuf stubs generated for it, do not travel to
that host); ``tests/`` checks it.  The product path never imports it.

What is restated, with the reference file:line each part follows:

* the wire message ``AllReducePayload`` / ``AllReduceResponse``
  (protos/distributed_inference.proto:85-96), built at run time from a descriptor so
  that the bytes on the wire are the reference's protobuf encoding;
* ``serialize_tensor`` / ``deserialize_tensor`` (engine/tensor_parallel/buffer_codec.py:27-69);
* ``DistributedCommunicator.all_reduce_sum`` / ``handle_incoming_allreduce`` /
  ``_broadcast_to_peers`` (engine/tensor_parallel/comm.py:55-154): the full tensor is
  sent to every peer over unary gRPC calls from a thread pool of ``max(4, 2 * world)``
  workers, the caller waits on an event for ``world - 1`` arrivals and sums
  ``local + peers`` in arrival order;
* the receiving servicer ``ExchangeAllReduce`` (engine/worker/worker_node.py:107-125) on
  a ``grpc.server`` with 16 threads and 100 MB message limits (worker_node.py:214-230);
* one rank's decoder layer in decode (engine/model/llama.py:48-76,
  engine/model/attention.py:135-233, engine/model/mlp.py:72-86): column-parallel q/k/v,
  RoPE, the per-sequence paged-KV store and gather, zero padding to the batch's longest
  context, ``repeat_kv``, batched scores / softmax / PV, row-parallel out_proj and
  down_proj each followed by the gRPC all-reduce, float32 throughout.

One process per rank (``multiprocessing`` spawn), each with an explicit torch CPU thread
count (cores // world), like the reference's one worker process per shard.
"""

from __future__ import annotations

import math
import os
import socket
import threading
import time
from concurrent import futures
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from oracle import decoder as od

SERVICE = "distributed_llm.WorkerService"
METHOD = f"/{SERVICE}/ExchangeAllReduce"
MAX_MSG = 100 * 1024 * 1024


# ------------------------------------------------------------------------------ wire format
_CLASSES = None


def wire_classes():
    """(AllReducePayload, AllReduceResponse) message classes with the reference's field numbers."""
    global _CLASSES
    if _CLASSES is not None:
        return _CLASSES
    from google.protobuf import descriptor_pb2, descriptor_pool, message_factory
    F = descriptor_pb2.FieldDescriptorProto
    fdp = descriptor_pb2.FileDescriptorProto(name="oracle_allreduce_wire.proto", package="distributed_llm",
                                             syntax="proto3")
    m = fdp.message_type.add(name="AllReducePayload")
    m.field.add(name="step_tag", number=1, type=F.TYPE_STRING, label=F.LABEL_OPTIONAL)
    m.field.add(name="sender_rank", number=2, type=F.TYPE_INT32, label=F.LABEL_OPTIONAL)
    m.field.add(name="shape", number=3, type=F.TYPE_INT64, label=F.LABEL_REPEATED)
    m.field.add(name="dtype", number=4, type=F.TYPE_STRING, label=F.LABEL_OPTIONAL)
    m.field.add(name="raw_tensor_data", number=5, type=F.TYPE_BYTES, label=F.LABEL_OPTIONAL)
    r = fdp.message_type.add(name="AllReduceResponse")
    r.field.add(name="success", number=1, type=F.TYPE_BOOL, label=F.LABEL_OPTIONAL)
    r.field.add(name="error_message", number=2, type=F.TYPE_STRING, label=F.LABEL_OPTIONAL)
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fdp)
    get = getattr(message_factory, "GetMessageClass", None)
    if get is None:  # older protobuf runtimes
        fac = message_factory.MessageFactory(pool)
        get = lambda d: fac.GetPrototype(d)  # noqa: E731
    _CLASSES = (get(pool.FindMessageTypeByName("distributed_llm.AllReducePayload")),
                get(pool.FindMessageTypeByName("distributed_llm.AllReduceResponse")))
    return _CLASSES


def serialize_tensor(t) -> Tuple[bytes, Tuple[int, ...], str]:
    """engine/tensor_parallel/buffer_codec.py:27-48: contiguous raw bytes, shape, dtype name."""
    arr = t.detach().contiguous().cpu().numpy() if hasattr(t, "detach") else np.ascontiguousarray(t)
    return arr.tobytes(), tuple(arr.shape), str(arr.dtype)


def deserialize_tensor(raw: bytes, shape: Sequence[int], dtype_str: str):
    """engine/tensor_parallel/buffer_codec.py:51-69: a writable torch tensor copied from the buffer."""
    import torch
    return torch.from_numpy(np.frombuffer(raw, dtype=np.dtype(dtype_str)).reshape(tuple(shape)).copy())


# ------------------------------------------------------------------------------ communicator
class GrpcAllReduce:
    """All-reduce(SUM) over unary gRPC calls between rank processes (engine/tensor_parallel/comm.py:27-166)."""

    def __init__(self, rank: int, world_size: int):
        self.rank = rank
        self.world_size = world_size
        self._executor = futures.ThreadPoolExecutor(max_workers=max(4, world_size * 2))
        self._lock = threading.Lock()
        self._events: Dict[Tuple[str, int], threading.Event] = {}
        self._payloads: Dict[Tuple[str, int], Dict[int, object]] = {}
        self._stubs: Dict[int, object] = {}
        self._channels: Dict[int, object] = {}
        self._server = None

    # worker_node.py:107-125 + serve_worker (214-230)
    def serve(self, port: int, host: str = "127.0.0.1"):
        import grpc
        Payload, Response = wire_classes()

        def exchange(request, context):
            try:
                t = deserialize_tensor(request.raw_tensor_data, tuple(request.shape), request.dtype)
                self.handle_incoming_allreduce(request.step_tag, request.sender_rank, t)
                return Response(success=True)
            except Exception as e:  # pragma: no cover - reported to the sender like the reference
                return Response(success=False, error_message=str(e))

        handler = grpc.method_handlers_generic_handler(SERVICE, {
            "ExchangeAllReduce": grpc.unary_unary_rpc_method_handler(
                exchange, request_deserializer=Payload.FromString, response_serializer=Response.SerializeToString)})
        self._server = grpc.server(futures.ThreadPoolExecutor(max_workers=16),
                                   options=[("grpc.max_receive_message_length", MAX_MSG),
                                            ("grpc.max_send_message_length", MAX_MSG)])
        self._server.add_generic_rpc_handlers((handler,))
        self._server.add_insecure_port(f"{host}:{port}")
        self._server.start()
        return self._server

    def connect(self, addresses: Sequence[str], ready_timeout: float = 60.0):
        """One insecure channel and stub per peer (worker_node.py:63-69); waits until each is ready."""
        import grpc
        Payload, Response = wire_classes()
        for r, addr in enumerate(addresses):
            if r == self.rank:
                continue
            ch = grpc.insecure_channel(addr, options=[("grpc.max_receive_message_length", MAX_MSG),
                                                      ("grpc.max_send_message_length", MAX_MSG)])
            grpc.channel_ready_future(ch).result(timeout=ready_timeout)
            self._channels[r] = ch
            self._stubs[r] = ch.unary_unary(METHOD, request_serializer=Payload.SerializeToString,
                                            response_deserializer=Response.FromString)

    def handle_incoming_allreduce(self, step_tag: str, sender_rank: int, tensor):
        """comm.py:55-70."""
        key = (step_tag, 0)
        with self._lock:
            self._payloads.setdefault(key, {})[sender_rank] = tensor
            if key in self._events and len(self._payloads[key]) >= self.world_size - 1:
                self._events[key].set()

    def all_reduce_sum(self, tensor, step_tag: str, timeout_sec: float = 15.0):
        """comm.py:72-118: send to every peer, wait for world-1 arrivals, local + peers (arrival order)."""
        if self.world_size <= 1:
            return tensor
        key = (step_tag, 0)
        with self._lock:
            self._payloads.setdefault(key, {})
            ev = threading.Event()
            self._events[key] = ev
            if len(self._payloads[key]) >= self.world_size - 1:
                ev.set()
        raw, shape, dt = serialize_tensor(tensor)
        self._broadcast(step_tag, raw, shape, dt, timeout_sec)
        if not ev.wait(timeout=timeout_sec):
            with self._lock:
                got = list(self._payloads.get(key, {}).keys())
            raise TimeoutError(f"[Rank {self.rank}] All-Reduce timeout on tag '{step_tag}'. "
                               f"Expected {self.world_size - 1} peers, received from ranks: {got}")
        with self._lock:
            peers = self._payloads.pop(key, {})
            self._events.pop(key, None)
        res = tensor.clone() if hasattr(tensor, "clone") else tensor.copy()
        for p in peers.values():
            res += p
        return res

    def _broadcast(self, step_tag, raw, shape, dt, timeout_sec):
        """comm.py:120-154: one payload message, sent to each peer from the thread pool."""
        Payload, _ = wire_classes()
        msg = Payload(step_tag=step_tag, sender_rank=self.rank, shape=list(shape), dtype=dt, raw_tensor_data=raw)

        def send(stub):
            try:
                stub(msg, timeout=timeout_sec)
            except Exception:
                pass  # the reference logs and carries on; the receiver's wait times out

        for r, stub in self._stubs.items():
            if r != self.rank:
                self._executor.submit(send, stub)

    def cleanup(self):
        for ch in self._channels.values():
            try:
                ch.close()
            except Exception:
                pass
        self._channels.clear()
        self._stubs.clear()
        self._executor.shutdown(wait=False)
        if self._server is not None:
            self._server.stop(grace=None)


# ------------------------------------------------------------------------------ one rank's layer
# The timed layer runs on torch's CPU kernels, as the reference does (its modules are
# torch CPU modules): numpy's single-threaded copies would make the gather / padding /
# repeat_kv steps several times slower than the reference's and overstate any speed-up.

def decode_attention_batched(q, k_new, v_new, positions, k_cache, v_cache, layer: int,
                             block_tables: Sequence[Sequence[int]], scale: float):
    """engine/model/attention.py:175-228 in torch, batched the way the reference does it.

    Per sequence: write the new token into its slot and gather its whole blocks, cut to
    the context (kv_cache.py:85-147); copy into zero-padded [B, max_len, kvh, hd] buffers
    without a mask; ``repeat_kv`` as an expand + reshape copy (attention.py:66-76); one
    batched score matmul, softmax over the padded length, one batched PV matmul.
    Equals ``oracle.decoder.decode_attention(..., compat_pad=True)``.
    q: [B, nq, hd]; k_new/v_new: [B, nkv, hd]; caches [L, NB, bs, nkv, hd]; returns [B, nq*hd].
    """
    import torch
    B, nq, hd = q.shape
    nkv = k_new.shape[1]
    rep = nq // nkv
    bs = k_cache.shape[2]
    ks, vs = [], []
    for b in range(B):
        pos = int(positions[b])
        blk, off = od.physical_slot(block_tables[b], pos, bs)
        k_cache[layer, blk, off] = k_new[b]
        v_cache[layer, blk, off] = v_new[b]
        ids = list(block_tables[b])
        ks.append(k_cache[layer, ids].reshape(-1, nkv, hd)[:pos + 1])
        vs.append(v_cache[layer, ids].reshape(-1, nkv, hd)[:pos + 1])
    L = max(k.shape[0] for k in ks)
    k_pad = torch.zeros(B, L, nkv, hd, dtype=q.dtype)
    v_pad = torch.zeros(B, L, nkv, hd, dtype=q.dtype)
    for b in range(B):
        k_pad[b, :ks[b].shape[0]] = ks[b]
        v_pad[b, :vs[b].shape[0]] = vs[b]
    k_rep = k_pad[:, :, :, None, :].expand(B, L, nkv, rep, hd).reshape(B, L, nq, hd)
    v_rep = v_pad[:, :, :, None, :].expand(B, L, nkv, rep, hd).reshape(B, L, nq, hd)
    s = torch.matmul(q[:, :, None, :], k_rep.transpose(1, 2).transpose(-2, -1)) * scale   # [B, nq, 1, L]
    p = torch.softmax(s, dim=-1)
    o = torch.matmul(p, v_rep.transpose(1, 2))                                            # [B, nq, 1, hd]
    return o.reshape(B, nq * hd)


def _fill(gen, shape, std):
    """Seeded float32 values tiled from a 1M-element draw (timing data; the values do not matter)."""
    import torch
    n = int(np.prod(shape))
    chunk = torch.randn(min(n, 1 << 20), generator=gen) * std
    reps = -(-n // chunk.numel())
    return chunk.repeat(reps)[:n].reshape(shape).contiguous()


class RankLayer:
    """Rank ``rank`` of ``world``: one decoder layer's weight shard and KV-pool shard, decode only.

    Weights follow the reference's layouts ([in, out] linears, engine/tensor_parallel/layers.py:55-61,
    :123-129); the pool is [1, blocks, 16, kv_heads/world, head_dim] float32 (kv_cache.py:70-80)
    with every sequence's block table a slice of one seeded permutation.
    """

    def __init__(self, hidden, heads, kv_heads, inter, rank, world, batch, ctx, seed, vocab_slice=0):
        import torch
        self.H, self.nq, self.nkv, self.I = hidden, heads // world, max(1, kv_heads // world), inter // world
        self.hd = hidden // heads
        self.rank, self.world = rank, world
        gen = torch.Generator().manual_seed(seed + 97 * rank)
        H, hd = hidden, self.hd
        self.w = {
            "q": _fill(gen, (H, self.nq * hd), 0.02), "k": _fill(gen, (H, self.nkv * hd), 0.02),
            "v": _fill(gen, (H, self.nkv * hd), 0.02), "o": _fill(gen, (self.nq * hd, H), 0.02),
            "g": _fill(gen, (H, self.I), 0.02), "u": _fill(gen, (H, self.I), 0.02),
            "d": _fill(gen, (self.I, H), 0.02),
            "n1": torch.ones(H), "n2": torch.ones(H),
        }
        bps = math.ceil((ctx + 64) / 16)
        self.k_cache = _fill(gen, (1, batch * bps, 16, self.nkv, hd), 1.0)
        self.v_cache = _fill(gen, (1, batch * bps, 16, self.nkv, hd), 1.0)
        perm = np.random.default_rng(seed).permutation(batch * bps)
        self.tables = [perm[b * bps:(b + 1) * bps].tolist() for b in range(batch)]
        cos, sin = od.rope_tables(hd, ctx + 64)
        self.cos, self.sin = torch.from_numpy(cos), torch.from_numpy(sin)
        self.lm = _fill(gen, (vocab_slice, H), 0.02) if vocab_slice else None

    @staticmethod
    def _rmsnorm(x, w, eps):
        """engine/tensor_parallel/layers.py:179-184."""
        import torch
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w

    def _rope(self, x, positions):
        """engine/model/attention.py:46-63 (rotate-half)."""
        import torch
        c = self.cos[positions].unsqueeze(-2)
        s = self.sin[positions].unsqueeze(-2)
        half = self.hd // 2
        return x * c + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * s

    def decode(self, h, positions, step_id: int, comm: GrpcAllReduce, eps: float = 1e-5):
        """engine/model/llama.py:48-76 for one rank; h: [B, 1, H] float32, positions [B, 1] int64."""
        import torch
        w = self.w
        B = h.shape[0]
        x = self._rmsnorm(h, w["n1"], eps)
        q = self._rope(torch.matmul(x, w["q"]).view(B, 1, self.nq, self.hd), positions)
        k = self._rope(torch.matmul(x, w["k"]).view(B, 1, self.nkv, self.hd), positions)
        v = torch.matmul(x, w["v"]).view(B, 1, self.nkv, self.hd)
        a = decode_attention_batched(q[:, 0], k[:, 0], v[:, 0], positions[:, 0], self.k_cache, self.v_cache, 0,
                                     self.tables, 1.0 / math.sqrt(self.hd))
        part = torch.matmul(a.view(B, 1, -1), w["o"])
        h = h + comm.all_reduce_sum(part, f"step_{step_id}_l0_attn")
        x2 = self._rmsnorm(h, w["n2"], eps)
        inter = torch.nn.functional.silu(torch.matmul(x2, w["g"])) * torch.matmul(x2, w["u"])
        return h + comm.all_reduce_sum(torch.matmul(inter, w["d"]), f"step_{step_id}_l0_mlp")

    def lm_slice(self, h):
        """The replicated lm_head (llama.py:121,168-170) on this rank's sampled vocabulary slice."""
        import torch
        return torch.matmul(self._rmsnorm(h[:, -1], self.w["n1"], 1e-5), self.lm.t())


# ------------------------------------------------------------------------------ processes
def free_ports(n: int) -> List[int]:
    socks, ports = [], []
    for _ in range(n):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        socks.append(s)
        ports.append(s.getsockname()[1])
    for s in socks:
        s.close()
    return ports


def cpu_threads() -> int:
    import torch
    return int(torch.get_num_threads())


def _decode_worker(rank, world, ports, threads, shape, batch, ctx, steps, warmup, seed, lm_frac, q):
    try:
        import torch
        torch.set_num_threads(threads)
        H, nq, nkv, inter, vocab, layers = shape
        vs = max(1, int(vocab * lm_frac))
        with torch.no_grad():
            layer = RankLayer(H, nq, nkv, inter, rank, world, batch, ctx, seed, vocab_slice=vs)
            comm = GrpcAllReduce(rank, world)
            if world > 1:
                comm.serve(ports[rank])
                comm.connect([f"127.0.0.1:{p}" for p in ports])
                comm.all_reduce_sum(torch.zeros(4), "ready", timeout_sec=120.0)
            h0 = torch.randn(batch, 1, H, generator=torch.Generator().manual_seed(seed + 5))
            recs = []
            for i in range(warmup + steps):
                pos = torch.full((batch, 1), ctx - 1 + i, dtype=torch.int64)
                t0 = time.perf_counter()
                h = layer.decode(h0, pos, i, comm)
                t1 = time.perf_counter()
                layer.lm_slice(h)
                t2 = time.perf_counter()
                if i >= warmup:
                    recs.append((t1 - t0, t2 - t1))
            comm.cleanup()
        q.put((rank, {"layer_s": [r[0] for r in recs], "lm_slice_s": [r[1] for r in recs], "vocab_slice": vs,
                      "threads": cpu_threads()}))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, {"error": repr(e)}))


def _spawn(target, world, cores, args, timeout):
    """Runs ``target(rank, world, args[0], threads, *args[1:], queue)`` in ``world`` spawned processes,
    each told to use ``threads = cores // world`` CPU threads; returns the per-rank result dicts."""
    import multiprocessing as mp
    threads = max(1, cores // world)
    keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
    saved = {k: os.environ.get(k) for k in keys}
    for k in keys:
        os.environ[k] = str(threads)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    try:
        procs = [ctx.Process(target=target, args=(r, world, args[0], threads) + tuple(args[1:]) + (q,))
                 for r in range(world)]
        for p in procs:
            p.start()
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    out: Dict[int, dict] = {}
    deadline = time.time() + timeout
    try:
        while len(out) < world:
            left = deadline - time.time()
            if left <= 0:
                raise TimeoutError(f"CPU rank processes did not finish within {timeout:.0f} s")
            r, d = q.get(timeout=left)
            if "error" in d:
                raise RuntimeError(f"CPU rank {r}: {d['error']}")
            out[r] = d
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    return [out[r] for r in range(world)], threads


def time_tp_decode(world: int, hidden: int, heads: int, kv_heads: int, inter: int, vocab: int, layers: int,
                   batch: int, ctx: int, steps: int, warmup: int, seed: int, cores: int,
                   lm_frac: float = 0.125, timeout: float = 1800.0) -> dict:
    """Decode ``batch`` sequences at context ``ctx`` through ONE decoder layer on ``world`` rank
    processes joined by the gRPC all-reduce, plus an ``lm_frac`` slice of the replicated lm_head,
    ``warmup + steps`` times.  Returns per-step seconds extrapolated to ``layers`` layers and the
    full lm_head (max over ranks), the sampled per-step wall times and the thread counts."""
    ports = free_ports(world)
    res, threads = _spawn(_decode_worker, world, cores,
                          (ports, (hidden, heads, kv_heads, inter, vocab, layers), batch, ctx, steps, warmup,
                           seed, lm_frac), timeout)
    vs = res[0]["vocab_slice"]
    step_s, sample_s = [], []
    for i in range(steps):
        lay = max(r["layer_s"][i] for r in res)
        lm = max(r["lm_slice_s"][i] for r in res)
        step_s.append(lay * layers + lm * vocab / vs)
        sample_s.append(lay + lm)
    return {"step_s": step_s, "sample_wall_s": sample_s, "threads_per_rank": threads,
            "threads_used": [r["threads"] for r in res], "vocab_slice": vs}


def _rowpar_worker(rank, world, ports, threads, tokens, hidden, inter, reps, seed, q):
    try:
        import torch
        torch.set_num_threads(threads)
        with torch.no_grad():
            comm = GrpcAllReduce(rank, world)
            comm.serve(ports[rank])
            comm.connect([f"127.0.0.1:{p}" for p in ports])
            comm.all_reduce_sum(torch.zeros(4), "ready", timeout_sec=120.0)
            gen = torch.Generator().manual_seed(seed + rank)
            K = inter // world
            w = _fill(gen, (K, hidden), 0.02)
            nw = torch.ones(hidden)
            rows = []
            for T in tokens:
                x = _fill(gen, (T, K), 1.0)
                res = _fill(gen, (T, hidden), 1.0)
                times = []
                for i in range(reps(T) + 1):
                    t0 = time.perf_counter()
                    part = torch.matmul(x, w)                                         # layers.py:147-152
                    s = comm.all_reduce_sum(part, f"rp_{T}_{i}", timeout_sec=600.0)   # layers.py:154-160
                    RankLayer._rmsnorm(res + s, nw, 1e-5)                             # llama.py:70-73
                    t1 = time.perf_counter()
                    if i > 0:
                        times.append(t1 - t0)
                rows.append(min(times))
            comm.cleanup()
        q.put((rank, {"s": rows, "threads": cpu_threads()}))
    except Exception as e:  # pragma: no cover
        q.put((rank, {"error": repr(e)}))


def _reps_for(T):
    return 3 if T <= 512 else 1


def time_row_parallel(world: int, tokens: Sequence[int], hidden: int, inter: int, seed: int, cores: int,
                      timeout: float = 1800.0) -> dict:
    """Row-parallel partial GEMM + gRPC all-reduce + residual + RMSNorm for each token count
    (float32, the reference's arithmetic); seconds per call, max over ranks."""
    ports = free_ports(world)
    res, threads = _spawn(_rowpar_worker, world, cores, (ports, list(tokens), hidden, inter, _reps_for, seed),
                          timeout)
    return {"s": [max(r["s"][i] for r in res) for i in range(len(tokens))], "threads_per_rank": threads,
            "threads_used": [r["threads"] for r in res]}
