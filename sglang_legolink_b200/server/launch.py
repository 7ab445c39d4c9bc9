"""Multi-GPU serving: ``--tp-size N`` (one model sharded over N GPUs) and
``--dp-size N`` (N replicas sharing one block directory), one process per GPU.

``python -m sglang_legolink_b200.server.http_server --tp-size 8 ...`` starts
the ranks itself (spawned children, rendezvous on 127.0.0.1); under
``torchrun`` the same flags use torchrun's ranks instead.

* **TP**: every rank loads its shard (fused NVLink TP boundary, or the
  collective library with ``--tp-comm nccl``); rank 0 serves HTTP and runs the
  scheduler over :class:`~sglang_legolink_b200.parallel.spmd.SPMDEngine`, the
  other ranks replay its engine calls.
* **DP**: every rank is a full replica (engine + scheduler + HTTP service) with
  its KV pool in symmetric memory and its compiled blocks published in the
  store-backed :class:`~sglang_legolink_b200.parallel.dp.BlockDirectory`, so a
  Link on any replica reads blocks compiled on another one over NVLink.
  Replicas ``r > 0`` listen on ``127.0.0.1:port + r``; rank 0 serves the public
  port through :class:`RouterService`.

Routing (:meth:`RouterService.pick`): a Compile of a key already published
goes to its owner (the owner's registry handles the duplicate); every other
request goes to the replica with the fewest requests in flight, ties broken
by the most referenced block tokens already resident there.  Key owners are
cached on the router (a stale entry only changes a preference).

Pipeline parallelism is refused, as the reference refuses a Link under PP
(``RT/pic_runtime.py:6279-6280``).  Reference DP/TP flags:
``RT/managers/scheduler.py:345-371``, ``scripts/serve_sglang.sh:44``.
"""

from __future__ import annotations

import http.client
import json
import faulthandler
import os
import signal
import socket
import threading
from collections import OrderedDict
from typing import Optional

from ..contract import ContractError
from ..runtime.scheduler import RequestRejected


class HTTPReplica:
    """A replica in another process, reached over its local HTTP port."""

    def __init__(self, host: str, port: int, timeout: float = 900.0):
        self.host, self.port, self.timeout = host, port, timeout

    def _conn(self):
        return http.client.HTTPConnection(self.host, self.port, timeout=self.timeout)

    def _request(self, method: str, path: str, body: Optional[dict] = None) -> dict:
        c = self._conn()
        try:
            data = json.dumps(body).encode() if body is not None else None
            c.request(method, path, body=data, headers={"Content-Type": "application/json"})
            r = c.getresponse()
            out = json.loads(r.read() or b"{}")
        finally:
            c.close()
        if r.status == 400:
            raise RequestRejected(out.get("message", "rejected"))
        if r.status != 200:
            raise RuntimeError(f"replica {self.port}: HTTP {r.status}: {out.get('message')}")
        return out

    def complete(self, payload: dict) -> dict:
        return self._request("POST", "/v1/chat/completions", dict(payload, stream=False))

    def stream(self, payload: dict):
        c = self._conn()
        try:
            c.request("POST", "/v1/chat/completions", body=json.dumps(dict(payload, stream=True)).encode(),
                      headers={"Content-Type": "application/json"})
            r = c.getresponse()
            if r.status != 200:
                out = json.loads(r.read() or b"{}")
                if r.status == 400:
                    raise RequestRejected(out.get("message", "rejected"))
                raise RuntimeError(f"replica {self.port}: HTTP {r.status}: {out.get('message')}")
            for line in r:
                line = line.strip()
                if not line.startswith(b"data: "):
                    continue
                data = line[6:]
                if data == b"[DONE]":
                    return
                yield json.loads(data)
        finally:
            c.close()

    def tokenize(self, payload: dict) -> dict:
        return self._request("POST", "/v1/tokenize", payload)

    def model_info(self) -> dict:
        return self._request("GET", "/model_info")


class RouterService:
    """The public service of a DP group: the :class:`RuntimeService` API over
    several replicas (in-process services or :class:`HTTPReplica`)."""

    def __init__(self, replicas: list, directory=None, model_name: Optional[str] = None, owner_cache: int = 65536):
        self.replicas = list(replicas)
        self.directory = directory
        self.model_name = model_name or getattr(self.replicas[0], "model_name", "default")
        self.inflight = [0] * len(self.replicas)
        self.routed = [0] * len(self.replicas)
        self._lock = threading.Lock()
        self._owners: OrderedDict = OrderedDict()
        self._owner_cap = owner_cache
        self._profiler = None

    # -------------------------------------------------------------- routing
    def _owner(self, key: str):
        """(owner replica, block tokens) of a published key, or None."""
        hit = self._owners.get(key)
        if hit is not None:
            self._owners.move_to_end(key)
            return hit
        if self.directory is None:
            return None
        b = self.directory.lookup(key)
        if b is None:
            return None
        hit = (int(b.owner), len(b.token_ids))
        self._owners[key] = hit
        if len(self._owners) > self._owner_cap:
            self._owners.popitem(last=False)
        return hit

    def pick(self, payload: dict, reserve: bool = False) -> int:
        """The replica for ``payload``; with ``reserve`` the choice is counted
        in flight under the same lock, so concurrent requests spread out."""
        n = len(self.replicas)
        sc, link = payload.get("sub_context"), payload.get("pic_link")
        if isinstance(sc, dict) and sc.get("cache_key") is not None:
            o = self._owner(str(sc["cache_key"]))
            if o is not None and 0 <= o[0] < n:
                if reserve:
                    self._enter(o[0])
                return o[0]
        local = [0] * n
        if isinstance(link, dict):
            for k in link.get("cache_keys") or ():
                o = self._owner(str(k))
                if o is not None and 0 <= o[0] < n:
                    local[o[0]] += o[1]
        with self._lock:
            r = min(range(n), key=lambda r: (self.inflight[r], -local[r], self.routed[r], r))
            if reserve:
                self.inflight[r] += 1
                self.routed[r] += 1
            return r

    def _enter(self, r: int) -> None:
        with self._lock:
            self.inflight[r] += 1
            self.routed[r] += 1

    def _leave(self, r: int) -> None:
        with self._lock:
            self.inflight[r] -= 1

    # ------------------------------------------------------------ API calls
    def complete(self, payload: dict) -> dict:
        r = self.pick(payload, reserve=True)
        try:
            out = self.replicas[r].complete(payload)
        finally:
            self._leave(r)
        out.setdefault("meta_info", {})["dp_replica"] = r
        return out

    def stream(self, payload: dict):
        r = self.pick(payload, reserve=True)
        try:
            for chunk in self.replicas[r].stream(payload):
                yield chunk
        finally:
            self._leave(r)

    def tokenize(self, payload: dict) -> dict:
        return self.replicas[0].tokenize(payload)

    def model_info(self) -> dict:
        info = dict(self.replicas[0].model_info())
        info["dp_size"] = len(self.replicas)
        info["dp_routed"] = list(self.routed)
        return info

    def warmup(self, block_tokens: int = 256, k: int = 16) -> dict:
        return self.replicas[0].warmup(block_tokens, k)


# ---------------------------------------------------------------- launching
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def check_parallel_args(tp: int, dp: int, pp: int) -> None:
    if pp != 1:
        raise ContractError("pipeline parallelism is not supported: a Link under PP is refused")
    if tp < 1 or dp < 1:
        raise ContractError("--tp-size and --dp-size must be >= 1")
    if tp > 1 and dp > 1:
        raise ContractError("--tp-size and --dp-size cannot both exceed 1")


def _build_rank(a, rank: int, world: int, local: int, ctrl=None):
    """(engine, tokenizer, model name, directory) of this rank."""
    import torch
    import torch.distributed as dist

    from ..host.tokenizer import HashTokenizer, HFTokenizer
    from ..models.config import get_config
    from ..models.qwen import QwenModel
    from ..runtime.engine import Engine

    cuda = torch.cuda.is_available() and not str(a.device).startswith("cpu")
    if cuda:
        torch.cuda.set_device(local)
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    dtype = torch.bfloat16 if cuda else torch.float32
    tp = a.tp_size
    comm, kw, directory = None, {}, None
    if tp > 1:
        if cuda and a.tp_comm == "fused":
            from ..parallel.tp_fused import FusedTPComm

            cfg0 = get_config(a.model) if not os.path.isdir(a.model) else None
            hidden = cfg0.hidden_size if cfg0 else json.load(open(os.path.join(a.model, "config.json")))["hidden_size"]
            comm = FusedTPComm(hidden, 16384, dev)
        else:
            from ..parallel.tp import NcclTPComm

            comm = NcclTPComm()
    tpr, tps = (rank, world) if tp > 1 else (0, 1)
    if os.path.isdir(a.model) and any(f.endswith(".safetensors") for f in os.listdir(a.model)):
        m = QwenModel.from_pretrained(a.model, device=dev, dtype=dtype, tp_rank=tpr, tp_size=tps, comm=comm)
    else:
        m = QwenModel.random_init(get_config(a.model), seed=a.seed, device=dev, dtype=dtype, tp_rank=tpr,
                                  tp_size=tps, comm=comm)
    if a.dp_size > 1:
        from ..parallel.dp import BlockDirectory

        directory = BlockDirectory(dist.distributed_c10d._get_default_store(), prefix="legolink-dp/", world=world)
        kw = dict(directory=directory, replica_rank=rank)
        if cuda:
            from ..parallel.dp import SharedKVPool

            per_page = 2 * m.cfg.num_layers * m.hkv * a.page_size * m.cfg.head_dim * 2
            free, _ = torch.cuda.mem_get_info(dev)
            pages = torch.tensor([max(64, int(free * 0.85 - (2 << 30)) // per_page)])
            dist.all_reduce(pages, op=dist.ReduceOp.MIN, group=ctrl)  # symmetric memory: one size on all ranks
            pages = int(pages)
            pool = SharedKVPool(m.cfg.num_layers, pages, m.hkv, a.page_size, m.cfg.head_dim, dtype, dev)
            kw.update(kv_pool=pool, peer_pools={r: pool.peer(r) for r in range(world) if r != rank})
    eng = Engine(m, page_size=a.page_size, max_context=a.context_length,
                 legolink_only=not a.allow_plain_generation, **kw)
    tok = HFTokenizer(a.tokenizer) if a.tokenizer else HashTokenizer(m.cfg.vocab_size, name=m.cfg.name)
    return eng, tok, m.cfg.name, directory


def rank_main(a, rank: int, world: int, local: int, ready=None) -> None:
    """One rank of a TP or DP server.  Returns when the server shuts down
    (rank 0: ``stop`` set; workers: rank 0's shutdown message)."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from ..parallel.spmd import SPMDEngine, control_group, worker_loop
    from ..runtime.scheduler import Scheduler
    from .http_server import RuntimeService, serve

    cuda = torch.cuda.is_available() and not str(a.device).startswith("cpu")
    if not dist.is_initialized():
        kw = {"device_id": torch.device("cuda", local)} if cuda else {}
        dist.init_process_group("nccl" if cuda else "gloo", timeout=timedelta(seconds=a.dist_timeout), **kw)
    ctrl = control_group()
    eng, tok, name, directory = _build_rank(a, rank, world, local, ctrl)
    stop = getattr(a, "stop_event", None) or threading.Event()
    if threading.current_thread() is threading.main_thread():
        # rank 0 turns SIGINT / SIGTERM into an orderly shutdown of every
        # rank; the others leave only on rank 0's message, between steps
        for sig in (signal.SIGINT, signal.SIGTERM):
            signal.signal(sig, (lambda *_: stop.set()) if rank == 0 else signal.SIG_IGN)
    try:
        if a.tp_size > 1:
            if rank != 0:
                worker_loop(eng, ctrl)
                return
            spmd = SPMDEngine(eng, ctrl)
            sch = Scheduler(spmd, legolink_only=False if a.allow_plain_generation else None)
            sch.start()
            svc = RuntimeService(sch, tok, model_name=name)
            try:
                if not a.skip_warmup:
                    print("warmup", svc.warmup(), flush=True)
                srv = serve(svc, a.host, a.port)
                print(f"serving TP={world} on http://{a.host}:{a.port}", flush=True)
                if ready is not None:
                    ready.put(a.port)
                _wait(stop)
                srv.shutdown()
            finally:
                sch.stop()
                spmd.shutdown()
            return
        # DP: every rank is a replica
        sch = Scheduler(eng, legolink_only=False if a.allow_plain_generation else None)
        sch.start()
        svc = RuntimeService(sch, tok, model_name=name)
        if not a.skip_warmup:
            print(f"replica {rank} warmup", svc.warmup(), flush=True)
        base = a.dp_base_port or a.port
        if rank != 0:
            srv = serve(svc, "127.0.0.1", base + rank)
        dist.barrier(group=ctrl)  # every replica listens before the router opens
        if rank == 0:
            reps = [svc] + [HTTPReplica("127.0.0.1", base + r) for r in range(1, world)]
            srv = serve(RouterService(reps, directory, model_name=name), a.host, a.port)
            print(f"serving DP={world} on http://{a.host}:{a.port}", flush=True)
            if ready is not None:
                ready.put(a.port)
        if rank == 0:
            _wait(stop)
            dist.broadcast_object_list(["stop"], src=0, group=ctrl)
        else:
            box = [None]
            dist.broadcast_object_list(box, src=0, group=ctrl)
        # a stop that stalls prints every thread's stack after 20 s
        faulthandler.dump_traceback_later(20, repeat=False)
        print(f"rank {rank}: stop received", flush=True)
        srv.shutdown()
        sch.stop()
        faulthandler.cancel_dump_traceback_later()
    finally:
        # a shutdown that stalls prints every thread's stack after a minute
        faulthandler.dump_traceback_later(60, repeat=False)
        print(f"rank {rank}: shutting down", flush=True)
        eng.release_graphs()
        dist.barrier(group=ctrl)
        print(f"rank {rank}: control barrier passed", flush=True)
        dist.destroy_process_group()
        faulthandler.cancel_dump_traceback_later()
        print(f"rank {rank}: stopped", flush=True)


def _wait(stop) -> None:
    while not stop.wait(0.5):
        pass


def _spawn_entry(rank: int, world: int, port: int, a) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    rank_main(a, rank, world, rank)


def launch(a) -> None:
    """Runs the ranks of ``a.tp_size * a.dp_size`` GPUs: under torchrun this
    process is one of them; otherwise spawn one child per rank."""
    check_parallel_args(a.tp_size, a.dp_size, a.pp_size)
    world = a.tp_size * a.dp_size
    if "WORLD_SIZE" in os.environ and int(os.environ["WORLD_SIZE"]) > 1:
        if int(os.environ["WORLD_SIZE"]) != world:
            raise ContractError(f"WORLD_SIZE={os.environ['WORLD_SIZE']} but tp*dp={world}")
        rank_main(a, int(os.environ["RANK"]), world, int(os.environ.get("LOCAL_RANK", os.environ["RANK"])))
        return
    import torch.multiprocessing as mp

    # the children inherit the ignored signals; rank 0 installs its own
    # handlers, and this process waits for every child to finish
    for sig in (signal.SIGINT, signal.SIGTERM):
        signal.signal(sig, signal.SIG_IGN)
    mp.start_processes(_spawn_entry, args=(world, _free_port(), a), nprocs=world, join=True,
                       start_method="spawn")
