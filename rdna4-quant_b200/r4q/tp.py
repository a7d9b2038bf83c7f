"""Tensor-parallel decode: weight sharding, the NVLink exchange comm and the
per-rank decode context.

The reference runs on one GPU only; this row-parallel split of the decode step
is new.  Per rank r of T (Megatron split):

* qkv rows: its H/T query heads, then its Hk/T key heads, then the same value
  heads (head-contiguous, so the grouped-query mapping stays local);
* gate_up rows: gate rows [r*I/T, (r+1)*I/T) then the same up rows, so the
  SiLU(gate)*up prologue of down_proj pairs the right halves;
* o_proj columns of its heads and down_proj columns of its intermediate slice
  (both multiples of 32, so no H32 block straddles two ranks); their fp32
  partial sums are all-reduced before the one fp16 rounding of the 1-GPU step;
* KV caches [B, Hk/T, max_seq, D] of its KV heads, lm_head rows of its
  vocabulary slice (logits are gathered on every rank);
* hidden state, norms and RoPE tables replicated.

The sharding helpers take the tuples of the oracle (('int4', packed, sz) |
('int8', w, s) | ('fp16', w)) or torch tensors alike, so the same code shards
the CPU oracle's model in the gloo tests and the device model on the GPU.
"""
from __future__ import annotations

import ctypes as C

import numpy as np


def _cat(parts):
    if isinstance(parts[0], np.ndarray):
        return np.ascontiguousarray(np.concatenate(parts, axis=0))
    import torch
    return torch.cat(parts, dim=0).contiguous()


def _contig(a):
    if isinstance(a, np.ndarray):
        return np.ascontiguousarray(a)
    return a.contiguous()


def fmt_of(w) -> str:
    """Weight precision from its storage type: uint8 packed -> int4, int8 -> int8, fp16."""
    name = str(w.dtype)
    if 'uint8' in name:
        return 'int4'
    if 'int8' in name:
        return 'int8'
    return 'fp16'


def shard_rows(lin, ranges):
    """Rows [r0, r1) of each range, concatenated, of a linear tuple."""
    kind = lin[0]
    out = [kind, _cat([lin[1][a:b] for a, b in ranges])]
    if kind != 'fp16':
        out.append(_cat([lin[2][a:b] for a, b in ranges]))
    return tuple(out)


def shard_cols(lin, k0, k1):
    """Input columns [k0, k1) (multiples of 32) of a linear tuple."""
    if k0 % 32 or k1 % 32:
        raise ValueError("column shards must be whole 32-blocks")
    kind = lin[0]
    if kind == 'int4':   # packed [N, K/2], (scale, zero) pairs [N, K/16]
        return ('int4', _contig(lin[1][:, k0 // 2:k1 // 2]), _contig(lin[2][:, k0 // 16:k1 // 16]))
    if kind == 'int8':   # int8 [N, K], scales [N, K/32]
        return ('int8', _contig(lin[1][:, k0:k1]), _contig(lin[2][:, k0 // 32:k1 // 32]))
    return ('fp16', _contig(lin[1][:, k0:k1]))


def check_split(cfg: dict, world: int, vocab: int | None = None):
    H, Hk, I = cfg['num_heads'], cfg['num_kv_heads'], cfg['intermediate_size']
    if H % world or Hk % world:
        raise ValueError(f"{H} query / {Hk} KV heads do not split over {world} ranks")
    if (I // world) % 128 or I % world:
        raise ValueError(f"intermediate {I} does not split into 128-multiples over {world} ranks")
    if vocab is not None and (vocab % world or (vocab // world) % 16):
        raise ValueError(f"vocabulary {vocab} does not split into 16-multiples over {world} ranks")


def local_cfg(cfg: dict, world: int) -> dict:
    """The per-rank model shape (heads and intermediate divided by world)."""
    out = dict(cfg)
    out['num_heads'] = cfg['num_heads'] // world
    out['num_kv_heads'] = cfg['num_kv_heads'] // world
    out['intermediate_size'] = cfg['intermediate_size'] // world
    return out


def shard_layer(layer: dict, cfg: dict, rank: int, world: int) -> dict:
    """Rank ``rank``'s shard of one layer in the oracle's dict format (keys
    qkv, o, gate_up, down, in_norm, post_norm, q_norm, k_norm)."""
    check_split(cfg, world)
    H, Hk, hd, I = cfg['num_heads'], cfg['num_kv_heads'], cfg['head_dim'], cfg['intermediate_size']
    hl, kl, il = H // world, Hk // world, I // world
    q0, k0, v0 = rank * hl * hd, H * hd + rank * kl * hd, (H + Hk) * hd + rank * kl * hd
    out = dict(layer)
    out['qkv'] = shard_rows(layer['qkv'], [(q0, q0 + hl * hd), (k0, k0 + kl * hd), (v0, v0 + kl * hd)])
    out['gate_up'] = shard_rows(layer['gate_up'], [(rank * il, (rank + 1) * il),
                                                   (I + rank * il, I + (rank + 1) * il)])
    out['o'] = shard_cols(layer['o'], rank * hl * hd, (rank + 1) * hl * hd)
    out['down'] = shard_cols(layer['down'], rank * il, (rank + 1) * il)
    return out


def shard_heads(cache, rank: int, world: int):
    """KV cache [B, Hk, max_seq, D] (or per-head scales [B, Hk]) -> this rank's heads."""
    axis = 1
    hk = cache.shape[axis]
    if hk % world:
        raise ValueError("KV heads do not split")
    n = hk // world
    return _contig(cache[:, rank * n:(rank + 1) * n])


def shard_lm(lm, rank: int, world: int):
    V = lm[1].shape[0]
    if V % world:
        raise ValueError("vocabulary does not split")
    n = V // world
    return shard_rows(lm, [(rank * n, (rank + 1) * n)])


def shard_decode_model(model: dict, cfg: dict, rank: int, world: int) -> dict:
    """Shard the device model of ``synth.build_decode_model`` (lists per
    projection, torch tensors) for rank ``rank``.  ``cfg`` uses the synth keys
    (num_heads, num_kv_heads, head_dim, intermediate, hidden, vocab)."""
    c = dict(num_heads=cfg['num_heads'], num_kv_heads=cfg['num_kv_heads'], head_dim=cfg['head_dim'],
             intermediate_size=cfg['intermediate'])
    check_split(c, world, int(model['lm_w'].shape[0]))
    out = {k: [] for k in ('qkv_w', 'qkv_s', 'o_w', 'o_s', 'gu_w', 'gu_s', 'down_w', 'down_s',
                           'k_caches', 'v_caches')}
    for li in range(len(model['qkv_w'])):
        ly = {}
        for name, key in (('qkv', 'qkv'), ('o', 'o'), ('gate_up', 'gu'), ('down', 'down')):
            w, s = model[key + '_w'][li], model[key + '_s'][li]
            f = fmt_of(w)
            ly[name] = (f, w) if f == 'fp16' else (f, w, s)
        sh = shard_layer(ly, c, rank, world)
        for name, key in (('qkv', 'qkv'), ('o', 'o'), ('gate_up', 'gu'), ('down', 'down')):
            out[key + '_w'].append(sh[name][1])
            out[key + '_s'].append(sh[name][2] if len(sh[name]) > 2 else None)
        out['k_caches'].append(shard_heads(model['k_caches'][li], rank, world))
        out['v_caches'].append(shard_heads(model['v_caches'][li], rank, world))
    for k in ('in_norm_w', 'post_norm_w', 'q_norm_w', 'k_norm_w', 'final_norm_w', 'rope_cos',
              'rope_sin', 'embed'):
        if k in model:
            out[k] = model[k]
    lm = ('fp16', model['lm_w']) if model.get('lm_s') is None else ('int4', model['lm_w'], model['lm_s'])
    sl = shard_lm(lm, rank, world)
    out['lm_w'], out['lm_s'] = sl[1], (sl[2] if len(sl) > 2 else None)
    out['vocab'] = int(model['lm_w'].shape[0])
    return out


# ---------------------------------------------------------------- device side
class Comm:
    """The NVLink exchange of one rank (r4q_comm_* in include/r4q.h).

    Creation is collective: every rank of ``group`` constructs its Comm with
    the same sizes; the CUDA IPC handles travel over torch.distributed (any
    backend)."""

    def __init__(self, rank: int, world: int, max_batch: int, hidden: int, vocab: int = 0,
                 sa_cap: int = 1 << 20, group=None):
        import torch.distributed as dist
        from . import lib as L
        self._L = L
        self.rank, self.world = rank, world
        self.max_batch, self.hidden, self.vocab = max_batch, hidden, vocab
        handle = (C.c_char * L.COMM_HANDLE_BYTES)()
        h = C.c_void_p()
        L.call("r4q_comm_create", rank, world, max_batch, hidden, vocab, sa_cap, C.byref(h), handle)
        self.handle = h
        hs = [None] * world
        if world > 1:
            dist.all_gather_object(hs, bytes(handle), group=group)
        else:
            hs = [bytes(handle)]
        blob = b"".join(hs)
        L.call("r4q_comm_open", h, blob)

    def allreduce_f32(self, x, out=None):
        """Sum of x over ranks (fp32, rank order); x is a CUDA fp32 tensor."""
        import torch
        from . import ops
        if x.dtype != torch.float32 or not x.is_cuda:
            raise TypeError("allreduce_f32 takes a CUDA float32 tensor")
        xc = x.contiguous()
        y = out if out is not None else torch.empty_like(xc)
        self._L.call("r4q_comm_allreduce_f32", self.handle, xc.data_ptr(), y.data_ptr(), xc.numel(),
                     ops.stream_handle(x.device))
        return y

    def status(self):
        """Raise R4QError if a device-side wait of this comm timed out."""
        self._L.call("r4q_comm_status", self.handle)

    def clear_status(self):
        self._L.call("r4q_comm_clear_status", self.handle)

    def close(self):
        if getattr(self, "handle", None):
            self._L.LIB.r4q_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TPDecoder:
    """One rank's decode step over its shard (``shard_decode_model`` output).

    ``cfg`` uses the synth keys (num_heads, num_kv_heads, head_dim, hidden,
    intermediate, rms_eps).  ``step`` returns the gathered logits
    [batch, vocab] (fp16, identical on every rank) or, with ``logits=False``,
    the replicated final hidden state."""

    def __init__(self, shard: dict, cfg: dict, comm: Comm, batch: int = 1):
        from . import decode
        self.comm, self.batch, self.hidden = comm, batch, int(cfg['hidden'])
        w = comm.world
        self.vocab = int(shard['vocab'])
        self.ctx = decode.get_context(
            shard['qkv_w'], shard['qkv_s'], shard['o_w'], shard['o_s'], shard['gu_w'], shard['gu_s'],
            shard['down_w'], shard['down_s'], shard['in_norm_w'], shard['post_norm_w'],
            shard['q_norm_w'], shard['k_norm_w'], shard['rope_cos'], shard['rope_sin'],
            cfg['num_heads'] // w, cfg['num_kv_heads'] // w, cfg['head_dim'], cfg['hidden'],
            cfg['intermediate'] // w, cfg['rms_eps'], shard['k_caches'], shard['v_caches'],
            shard['final_norm_w'], shard['lm_w'], shard['lm_s'], self.vocab // w, batch=batch,
            comm=comm)

    def loop(self, embed, h, start_pos: int, num_tokens: int, use_graph: bool = True):
        """Greedy tokens [num_tokens, batch] (device int64), identical on every rank."""
        return self.ctx.loop(embed, h.reshape(self.batch, self.hidden), start_pos, num_tokens, use_graph)

    def step(self, h, pos: int, logits: bool = True, out=None, use_graph: bool = True):
        import torch
        h2 = h.reshape(self.batch, self.hidden)
        if logits:
            y = out if out is not None else torch.empty(self.batch, self.vocab, dtype=torch.float16,
                                                        device=h.device)
            self.ctx.step(h2, pos, logits_out=y, use_graph=use_graph)
        else:
            y = out if out is not None else torch.empty_like(h2)
            self.ctx.step(h2, pos, hidden_out=y, use_graph=use_graph)
        return y
