"""Fused peer-memory replacements of the NCCL collectives (the product path).

* ``FusedUlysses`` — Ulysses sequence parallelism with
  (1) RMS qk-norm + RoPE + head-scatter all-to-all in one kernel (qkv_scatter),
  (2) a bounded flag barrier,
  (3) attention on the gathered full sequence whose epilogue stores each output
      row into the owning rank's O buffer (the inverse all-to-all),
  (4) a second barrier before the output projection reads O.
* ``FusedCFG`` — CFG parallelism: each rank writes its branch prediction into
  its heap; one kernel signals the partner, waits (bounded), reads the partner's
  prediction over NVLink and applies guidance + the UniPC/Euler update.
Reference collectives replaced: usp.py:207-270/:368-381 (all_to_all_single) and
xdit/wan.py:187-203 (prediction all_gather).
"""
from __future__ import annotations

import math

import torch

from ..ops._ext import ext, kernel, status_word
from .symm import PeerGroup, SymmetricHeap

CH_SP, CH_CFG, CH_GATHER, CH_USP_ADDR, CH_RING = 0, 1, 2, 3, 8


class FusedUlysses:
    def __init__(self, heap: SymmetricHeap, members: tuple, seq_local: int, heads: int, head_dim: int,
                 batch: int, gather_cols: int = 64):
        self.group = PeerGroup(heap, members, CH_SP)
        self.gather_group = PeerGroup(heap, members, CH_GATHER)
        self.heap = heap
        self.sp_size = self.group.size
        self.sp_rank = self.group.rank
        self.seq_local = seq_local
        self.heads = heads
        self.head_dim = head_dim
        self.batch = batch
        P = self.sp_size
        hl = heads // P
        S = seq_local * P
        self.recv_off, self.recv = heap.alloc_view((batch * S, 3 * hl * head_dim))
        self.o_off, self.o = heap.alloc_view((batch * seq_local, heads * head_dim))
        self.gather_off, self.gathered = heap.alloc_view((P * batch * seq_local, gather_cols))
        self.gather_cols = gather_cols

    def fused_qkv_attention(self, qkv, wq, wk, eps, cos_full, sin_full, heads, batch, seq_local):
        assert batch == self.batch and seq_local == self.seq_local and heads == self.heads
        st = status_word(qkv.device)
        r, bases, tmo = self.group.args()
        kernel("qkv_scatter")(qkv, wq, wk, float(eps), cos_full, sin_full, seq_local, heads, self.head_dim, r, bases,
                          tmo, self.recv_off, 0)
        self.group.barrier(st)
        hl = heads // self.sp_size
        w = hl * self.head_dim
        q, k, v = self.recv[:, :w], self.recv[:, w:2 * w], self.recv[:, 2 * w:]
        kernel("attention_scatter")(q, k, v, batch, seq_local * self.sp_size, hl, self.head_dim,
                                1.0 / math.sqrt(self.head_dim), r, bases, tmo, self.o_off, seq_local,
                                self.sp_rank * hl, heads * self.head_dim, st, [], [])
        self.group.barrier(st)
        return self.o

    def gather_sequence(self, y, batch, seq_local):
        if y.shape[1] != self.gather_cols:
            raise ValueError("gather width differs from the reserved buffer")
        r, bases, tmo = self.gather_group.args()
        kernel("allgather_rows")(y.contiguous(), self.gather_off, r, bases, tmo)
        self.gather_group.barrier(status_word(y.device))
        P = self.sp_size
        return self.gathered.view(P, batch, seq_local, -1).permute(1, 0, 2, 3).reshape(batch * P * seq_local, -1)


class FusedUSP(FusedUlysses):
    """Ulysses x ring (2D USP): heads exchanged inside the U-group, keys/values of the ring
    peers read in place by the attention mainloop (multi-source TMA over peer memory, no
    multicast).  With an active INT8 ring codec the peers' chunks come instead as int8
    packets pushed into this rank's heap (``ring_quant_push``) and decoded locally
    (``ring_dequant``) before the same attention kernel reads them."""

    def __init__(self, heap: SymmetricHeap, sp_members: tuple, ring: int, seq_local: int, heads: int, head_dim: int,
                 batch: int, gather_cols: int = 64, codec=None):
        P = len(sp_members)
        U = P // ring
        m = sp_members.index(heap.rank)
        self.r, self.u, self.U, self.R = m // U, m % U, U, ring
        self.sp_group = PeerGroup(heap, sp_members, CH_SP)
        self.gather_group = PeerGroup(heap, sp_members, CH_GATHER)
        self.ugroup = PeerGroup(heap, sp_members[self.r * U:(self.r + 1) * U], CH_USP_ADDR)
        self.ring_members = [sp_members[rr * U + self.u] for rr in range(ring)]
        self.heap = heap
        self.sp_size, self.sp_rank = P, m
        self.seq_local, self.heads, self.head_dim, self.batch = seq_local, heads, head_dim, batch
        hl = heads // U
        chunk = seq_local * U  # tokens of one ring chunk
        self.recv_off, self.recv = heap.alloc_view((batch * chunk, 3 * hl * head_dim))
        self.o_off, self.o = heap.alloc_view((batch * seq_local, heads * head_dim))
        self.gather_off, self.gathered = heap.alloc_view((P * batch * seq_local, gather_cols))
        self.gather_cols = gather_cols
        self.group = self.sp_group
        self.codec = codec
        if codec is not None:
            # INT8 ring transport: one packet slot per ring source in every ring member's heap,
            # and local bf16 buffers (receive-buffer layout) for the decoded peer chunks
            rows = batch * chunk
            self.ring_group = PeerGroup(heap, tuple(self.ring_members), CH_RING)
            self.slot_bytes = int(ext().ring_slot_bytes(rows, hl, head_dim))
            self.slot_off = heap.alloc(ring * self.slot_bytes, align=256)
            self.decoded = torch.empty((ring - 1, rows, 3 * hl * head_dim), device=heap.device, dtype=torch.bfloat16)

    def set_step(self, step: int, total_steps: int):
        if self.codec is not None:
            self.codec.set_step(step, total_steps)

    def _int8_ring_sources(self, w, st):
        """Quantize this rank's K/V chunk into every ring peer's slot, then decode the peers'
        slots locally; returns the decoded chunks' K and V addresses in ring order."""
        rg = self.ring_group
        r, bases, tmo = rg.args()
        hl = self.heads // self.U
        kernel("ring_quant_push")(self.recv[:, w:], hl, self.head_dim, r, self.slot_off, self.slot_bytes, r, bases,
                                  tmo)
        rg.barrier(st)
        k_extra, v_extra = [], []
        others = [i for i in range(self.R) if i != r]
        for buf, src in zip(self.decoded, others):
            kernel("ring_dequant")(buf, hl, self.head_dim, src, self.slot_off, self.slot_bytes, r, bases, tmo)
            k_extra.append(buf.data_ptr() + w * 2)
            v_extra.append(buf.data_ptr() + 2 * w * 2)
        self.codec.account(self.recv.shape[0], hl, self.head_dim, True, self.R - 1)
        return k_extra, v_extra

    def fused_qkv_attention(self, qkv, wq, wk, eps, cos_full, sin_full, heads, batch, seq_local):
        st = status_word(qkv.device)
        ur, ub, utmo = self.ugroup.args()
        chunk = seq_local * self.U
        kernel("qkv_scatter")(qkv, wq, wk, float(eps), cos_full, sin_full, seq_local, heads, self.head_dim, ur, ub,
                              utmo, self.recv_off, self.r * chunk)
        self.sp_group.barrier(st)
        hl = heads // self.U
        w = hl * self.head_dim
        q, k, v = self.recv[:, :w], self.recv[:, w:2 * w], self.recv[:, 2 * w:]
        if self.codec is not None and self.codec.active:
            k_extra, v_extra = self._int8_ring_sources(w, st)
        else:
            # bf16: the attention mainloop reads the ring peers' chunks in place (TMA, no multicast)
            peers = [m for m in self.ring_members if m != self.heap.rank]
            k_extra = [self.heap.bases[m] + self.recv_off + w * 2 for m in peers]
            v_extra = [self.heap.bases[m] + self.recv_off + 2 * w * 2 for m in peers]
            if self.codec is not None:
                self.codec.account(self.recv.shape[0], hl, self.head_dim, False, self.R - 1)
        kernel("attention_scatter")(q, k, v, batch, chunk, hl, self.head_dim, 1.0 / math.sqrt(self.head_dim), ur, ub,
                                utmo, self.o_off, seq_local, self.u * hl, heads * self.head_dim, st, k_extra,
                                v_extra)
        self.sp_group.barrier(st)
        return self.o


class FusedCFG:
    """CFG pair over peer memory; cfg_rank 0 computes the conditional branch."""

    def __init__(self, heap: SymmetricHeap, members: tuple, numel: int):
        self.group = PeerGroup(heap, members, CH_CFG)
        self.heap = heap
        self.cfg_size = 2
        self.cfg_rank = self.group.rank
        self.numel = numel
        # double-buffered prediction slots (parity of the exchange epoch)
        self.slots = [heap.alloc_view((numel,)) for _ in range(2)]
        self.calls = 0

    def exchange(self, mine):  # pragma: no cover - the fused step never exchanges separately
        raise RuntimeError("FusedCFG applies guidance inside the exchange kernel")

    def fused_step(self, scheduler, sample: torch.Tensor, mine: torch.Tensor, guidance: float,
                   delta_out: torch.Tensor | None = None):
        """Exchange + guidance + solver update in one kernel; ``delta_out`` (fp32, latent size)
        also receives cond - uncond, which late-step CFG folding reuses."""
        n = mine.numel()
        if n > self.numel:
            raise ValueError(f"prediction of {n} elements exceeds the reserved CFG slot ({self.numel})")
        slot_off, slot = self.slots[self.calls & 1]
        slot = slot[:n]
        self.calls += 1
        slot.copy_(mine.reshape(-1))
        r, bases, tmo = self.group.args()
        epoch = self.heap.next_epoch(self.group.channel)
        st = status_word(sample.device)

        def step_kernel(cond, uncond, g, x, sigma, corr, pred, x0_out=None, last_out=None):
            c = corr or {}
            kernel("cfg_step_peer")(
                slot, slot_off, self.cfg_rank, float(g), x, float(sigma), corr is not None, c.get("last"),
                float(c.get("last_coef", 0.0)), float(c.get("x0_coef", 0.0)), list(c.get("hist", [])),
                [float(v) for v in c.get("hist_coef", [])], float(pred.get("x", 1.0)), float(pred.get("x0", 0.0)),
                float(pred.get("v", 0.0)), list(pred.get("hist", [])), [float(v) for v in pred.get("hist_coef", [])],
                x0_out, last_out, r, bases, tmo, self.group.channel, epoch, st, delta_out)
            return x

        return scheduler.step(sample, mine.reshape(-1), None, guidance, kernel=step_kernel)


def upgrade(layout, rank, device, pctx, cfg_plan, sp_groups, cfg_groups, seq_local=None, cfg=None,
            heap_bytes: int | None = None, pred_numel: int | None = None, codec=None):
    """Replace the NCCL plans of ``build_parallel`` by fused peer-memory ones (same layout)."""
    if device.type != "cuda" or cfg is None or seq_local is None:
        return pctx, cfg_plan
    form = layout.form
    batch = 1 if form.cfg == 2 else 2
    P = form.sp
    hl = cfg.heads // P
    need = 0
    if P > 1:
        hl = cfg.heads // form.ulysses
        need += batch * seq_local * form.ulysses * 3 * hl * cfg.head_dim * 2 + batch * seq_local * cfg.dim * 2
        need += P * batch * seq_local * cfg.out_channels * 4 * 2
        if form.ring > 1 and codec is not None:
            need += form.ring * int(ext().ring_slot_bytes(batch * seq_local * form.ulysses, hl, cfg.head_dim)) + 4096
    pred_numel = pred_numel or 8 * 1024 * 1024
    need += 2 * pred_numel * 2  # double-buffered bf16 prediction slots
    from .runtime import group_for
    # one heap over the layout's ranks; heap index = position in the sorted rank list
    heap = SymmetricHeap(heap_bytes or int(need * 1.2) + (64 << 20), device, group=group_for(layout.ranks))
    hidx = {g: i for i, g in enumerate(sorted(layout.ranks))}

    def h(ranks):
        return tuple(hidx[r] for r in ranks)
    if P > 1 and form.ring > 1:
        pctx = FusedUSP(heap, h(layout.sp_ranks(rank)), form.ring, seq_local, cfg.heads, cfg.head_dim, batch,
                        gather_cols=cfg.out_channels * math.prod(cfg.patch), codec=codec)
    elif P > 1:
        pctx = FusedUlysses(heap, h(layout.sp_ranks(rank)), seq_local, cfg.heads, cfg.head_dim, batch,
                            gather_cols=cfg.out_channels * math.prod(cfg.patch))
    if form.cfg == 2:
        partner = layout.cfg_partner(rank)
        members = (rank, partner) if layout.cfg_role(rank) == 0 else (partner, rank)
        cfg_plan = FusedCFG(heap, h(members), numel=pred_numel)
    return pctx, cfg_plan


class PeerHalo:
    """Patch-parallel VAE halo exchange over peer memory (drop-in for ``vae.PatchParallel``).

    ``pad``: this rank's first slice is stored straight into the left neighbour's right-halo
    buffer and its last slice into the right neighbour's left-halo buffer (strided_put over
    NVLink), one bounded barrier, then the slab is completed from the local halo buffers.
    ``gather``/``local`` (mid-block attention at latent resolution) reuse the NCCL baseline.
    """

    def __init__(self, heap: SymmetricHeap, members: tuple, axis: int = 4, max_halo_elems: int = 4 << 20,
                 channel: int = 4, baseline=None):
        self.group = PeerGroup(heap, members, channel)
        self.heap = heap
        self.size, self.rank, self.axis = self.group.size, self.group.rank, axis
        self.max_elems = max_halo_elems
        # two slots per side, alternating per exchange: a neighbour's next put (slot k+1) can
        # land before this rank has read slot k, never before it read slot k-1
        self.left_off = [heap.alloc(max_halo_elems * 4) for _ in range(2)]
        self.right_off = [heap.alloc(max_halo_elems * 4) for _ in range(2)]
        self.calls = 0
        self.baseline = baseline

    def pad(self, x):
        a = self.axis
        n = x.shape[a]
        first = x.narrow(a, 0, 1)
        last = x.narrow(a, n - 1, 1)
        shape = list(first.shape)
        numel = first.numel()
        if numel > self.max_elems:
            raise ValueError("halo slice exceeds the reserved buffer")
        r, bases, tmo = self.group.args()
        slot = self.calls & 1
        self.calls += 1
        sq = lambda t: t.squeeze(a)  # 4-D strided view of the slice
        if self.rank > 0:
            kernel("strided_put")(sq(first), self.rank - 1, self.right_off[slot], r, bases, tmo)
        if self.rank < self.size - 1:
            kernel("strided_put")(sq(last), self.rank + 1, self.left_off[slot], r, bases, tmo)
        self.group.barrier(status_word(x.device))
        esz = x.element_size()
        view = lambda off: self.heap.tensor[off:off + numel * esz].view(x.dtype).view(shape)
        left = view(self.left_off[slot]) if self.rank > 0 else torch.zeros_like(first)
        right = view(self.right_off[slot]) if self.rank < self.size - 1 else torch.zeros_like(last)
        return torch.cat([left, x, right], dim=a)

    def gather(self, x):
        return self.baseline.gather(x)

    def local(self, x):
        return self.baseline.local(x)
