"""Expert parallelism: one process per GPU, experts sharded by id.

The reference computes every routed expert of a token in one process
(run_batch + the rank-ordered combine, src/lib/tlm_model.c:900-938,
:1029-1036). Here the experts of each layer are split over the N GPUs of a
torch.distributed group: expert e is owned by GPU floor(e * N / E). Each
GPU is the home of its own batch of tokens (its sequences); one layer call
runs

    dispatch   home: route + quantise its tokens, one record per
               (token, rank) pair grouped by owner           (C ABI, CUDA)
    exchange   record counts (kept on the device; one host read
               of both directions), then the records         (all-to-all)
    experts    owner: the expert FFN of every received record (C ABI, CUDA)
    exchange   expert output rows back, in record order      (all-to-all)
    combine    home: ffn[t] = sum_r w[t, r] * eo[t, r], ascending r
                                                             (C ABI, CUDA)

Every (token, expert) output row is computed exactly as on one GPU and the
combine keeps rank order, so the result is bit-identical for any N.

The compute steps go through a backend object with the MoeContext methods
ep_record_bytes / ep_dispatch / ep_experts / ep_combine; the product
backend is a MoeContext on the process's GPU, switched onto torch's current
stream so that its kernels and the collectives are ordered. The exchange
uses torch.distributed.all_to_all_single (NCCL on GPUs).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def owner(expert: int, n_ranks: int, n_experts: int) -> int:
    """The GPU that owns an expert: floor(e * N / E)."""
    return expert * n_ranks // n_experts


def owned_range(rank: int, n_ranks: int, n_experts: int) -> tuple[int, int]:
    """[lo, hi) of the experts a GPU owns."""
    lo = -(-rank * n_experts // n_ranks)
    hi = -(-(rank + 1) * n_experts // n_ranks)
    return lo, hi


class ExpertParallel:
    """Expert-parallel routed-expert FFN of one process's token batch."""

    def __init__(self, backend, d_model: int, n_experts: int, top_k: int, group=None,
                 device: torch.device | None = None):
        self.b = backend
        self.D = d_model
        self.E = n_experts
        self.k = top_k
        self.group = group
        self.n_ranks = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device if device is not None else torch.device("cpu")
        if self.device.type == "cuda" and hasattr(backend, "set_stream"):
            # the backend's kernels and the collectives share torch's stream
            backend.set_stream(torch.cuda.current_stream(self.device))
        self.RB = int(backend.ep_record_bytes)
        self.lo, self.hi = owned_range(self.rank, self.n_ranks, n_experts)
        self._send = self._perm = self._w = self._back = None
        self._recv = self._eo = None

    def _grow(self, n_tok: int) -> None:
        npair = max(n_tok * self.k, 1)
        if self._send is None or self._send.shape[0] < npair:
            dev = self.device
            self._send = torch.empty((npair, self.RB), dtype=torch.uint8, device=dev)
            self._perm = torch.empty(npair, dtype=torch.int32, device=dev)
            self._w = torch.empty(npair, dtype=torch.float32, device=dev)
            self._back = torch.empty((npair, self.D), dtype=torch.float32, device=dev)

    def _grow_recv(self, n_rec: int) -> None:
        n = max(n_rec, 1)
        if self._recv is None or self._recv.shape[0] < n:
            self._recv = torch.empty((n, self.RB), dtype=torch.uint8, device=self.device)
            self._eo = torch.empty((n, self.D), dtype=torch.float32, device=self.device)

    def _a2a(self, out, inp, out_splits, in_splits) -> None:
        if self.n_ranks == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def ffn_batch(self, layer: int, x: torch.Tensor, logits: torch.Tensor, ffn: torch.Tensor,
                  check: bool = True) -> dict:
        """x [n][D], logits [n][E] -> ffn [n][D] for this process's n tokens
        (n may be 0; every rank must call with the same layer). Returns the
        record counts {"sent": [per owner], "received": [per home]}.

        Errors the kernels raise on the device (a tensor-core wait that
        expired, a received record naming an expert this GPU does not own)
        are raised by this call: those of earlier calls once the counts are
        back on the host, those of this call at the end when `check` is
        true (one more stream synchronisation). A caller running many layers
        back to back may pass check=False for all but the last layer of a
        step: an error of layer l is then raised by the call for layer l+1."""
        n = int(x.shape[0])
        self._grow(n)
        npair = n * self.k
        send = self._send[:npair]
        # counts: sent[d] records go to owner d; received[s] arrive from home s
        if self.device.type == "cuda" and hasattr(self.b, "ep_dispatch_async"):
            # counts stay on the device through their exchange; one host read
            # of both directions sizes the record exchange
            sc = torch.empty(self.n_ranks, dtype=torch.int64, device=self.device)
            self.b.ep_dispatch_async(layer, x, logits, self.n_ranks, send, self._perm, self._w, sc)
            rc = torch.empty_like(sc)
            self._a2a(rc, sc, None, None)
            both = torch.cat([sc, rc]).tolist()
            sent, received = both[:self.n_ranks], both[self.n_ranks:]
            # the stream is idle now: report what earlier kernels flagged
            self.b.check()
        else:
            sent = self.b.ep_dispatch(layer, x, logits, self.n_ranks, send, self._perm, self._w)
            sc = torch.tensor(sent, dtype=torch.int64, device=self.device)
            rc = torch.empty_like(sc)
            self._a2a(rc, sc, None, None)
            received = [int(v) for v in rc.tolist()]
        if sum(sent) != npair:
            raise RuntimeError(f"dispatch wrote {sum(sent)} records for {npair} pairs")
        n_rec = sum(received)
        self._grow_recv(n_rec)
        recv = self._recv[:n_rec]
        self._a2a(recv, send, received, sent)
        eo = self._eo[:n_rec]
        self.b.ep_experts(layer, self.lo, self.hi, n_rec, recv, eo)
        back = self._back[:npair]
        self._a2a(back, eo, sent, received)
        self.b.ep_combine(n, back, self._perm, self._w, ffn)
        if check and hasattr(self.b, "check"):
            self.b.check()
        return {"sent": sent, "received": received}


class PeerExpertParallel:
    """ExpertParallel with the exchange done by the library over peer memory
    (tlmg_ep_open / tlmg_ep_layer, include/tlmg.h): each rank maps every
    peer's exchange buffer through CUDA IPC, and one layer call queues
    dispatch, the owner's experts, the return of the rows and the combine
    on the stream, ordered by two bounded device barriers over peer flags:
    no host synchronisation and no collective in the data path. Results are
    bit-identical to ExpertParallel and to the one-GPU batched call.

    torch.distributed is used once, to exchange the buffers' IPC handles.
    All ranks must sit on GPUs of one node."""

    def __init__(self, backend, d_model: int, n_experts: int, top_k: int, max_tok: int, group=None,
                 device: torch.device | None = None):
        self.b = backend
        self.D, self.E, self.k = d_model, n_experts, top_k
        self.group = group
        self.n_ranks = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.max_tok = max_tok
        if hasattr(backend, "set_stream"):
            backend.set_stream(torch.cuda.current_stream(self.device))
        self.lo, self.hi = owned_range(self.rank, self.n_ranks, n_experts)
        mine = backend.ep_open(self.rank, self.n_ranks, max_tok)
        handles = [mine]
        if self.n_ranks > 1:
            handles = [None] * self.n_ranks
            dist.all_gather_object(handles, mine, group=self.group)
        backend.ep_connect(handles)
        torch.cuda.synchronize(self.device)
        if self.n_ranks > 1:
            dist.barrier(group=self.group)   # every peer mapped before the first device barrier

    def ffn_batch(self, layer: int, x: torch.Tensor, logits: torch.Tensor, ffn: torch.Tensor,
                  check: bool = True, ids: torch.Tensor | None = None, w: torch.Tensor | None = None) -> None:
        """x [n][D], logits [n][E] -> ffn [n][D] for this process's n tokens
        (n <= max_tok, may be 0; every rank calls with the same layers in
        the same order). With `check` the call waits for the stream and
        raises what the kernels flagged (a barrier that gave up, a
        tensor-core wait that expired); otherwise that shows at a later
        check."""
        if x.shape[0] > self.max_tok:
            raise ValueError(f"{x.shape[0]} tokens; the exchange was opened for {self.max_tok}")
        self.b.ep_layer(layer, x, logits, ffn, ids, w)
        if check:
            self.b.check()

    def close(self) -> None:
        self.b.ep_close()
