"""DiT denoiser forward on the sm_100a kernels.

DiTEngine takes a reference-shaped DiffusionTransformer (sa3_b200.modules,
same parameter names as stable_audio_3/models/dit.py) and runs
DiffusionTransformer.forward (dit.py:345-643) -> _forward (dit.py:179-309) ->
ContinuousTransformer.forward (transformer.py:1161-1272) -> TransformerBlock.forward
(transformer.py:996-1049) with every hot op in libsa3b200.so:

  per block (token rows [B*N, D], N = L + memory tokens):
    RMSNorm+adaLN modulate (+FP8 quant)   -> to_qkv GEMM with qk RMSNorm + RoPE in its epilogue
    -> windowed (differential) attention   -> to_out GEMM with gate*sigmoid(1-g)+residual epilogue
    cross: RMSNorm (+quant) -> to_q GEMM (+q-norm epilogue) ; ctx -> to_kv GEMM (+k-norm epilogue)
           -> full attention over the context -> to_out GEMM with residual epilogue
    local cond: Linear+SiLU GEMM -> Linear GEMM adding into rows 64.. (left pad) of the stream
    FF: RMSNorm+modulate (+quant) -> GLU.proj GEMM with SwiGLU epilogue (+amax) (-> quant)
        -> linear_out GEMM with gate*sigmoid(1-g)+residual epilogue

Exact rewrites of the reference:
  * preprocess_conv (1x1, +x) is folded into project_in: W_in (I + W_pre);
    postprocess_conv (1x1, +y) into project_out: (I + W_post) W_out.
  * GLU.proj rows are interleaved in blocks of 128 so the SwiGLU fuses into the GEMM epilogue.
  * local_add_cond's 257 channels are zero-padded to 264 (16-byte rows for TMA).
The residual stream (the token rows every block adds into) and the final
projection are kept in fp32; GEMM operands and the other activations are bf16
(or e4m3). The timestep is kept in fp32 through ExpoFourierFeatures (the
reference's bf16 path rounds it first); the CFG / APG combine runs in fp32.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np
from typing import Dict, Optional

import torch

from . import ops
from . import _lib
from . import gptq as _gptq
from . import seqsplit as _seqsplit
from .quant import interleave_swiglu_rows, quantize_weight_e4m3, swiglu_interleave_index

QUANT_SUFFIXES = ("self_attn.to_qkv", "self_attn.to_out", "cross_attn.to_q", "cross_attn.to_kv",
                  "cross_attn.to_out", "ff.ff.0.proj", "ff.ff.2")

# Byte budget of the batched first local-conditioning layer's output (every block's SiLU(W1 c + b1) for all
# latent rows); larger packed batches compute it block by block.
_LOCAL_ALL_MAX_BYTES = 4 << 30

# FP8 norms outside a sequence split run both passes as one launch (grid barrier); SA3_NORM_FUSED=0 in the
# environment selects the two launches (the same bytes)
_NORM_ONE_LAUNCH = os.environ.get("SA3_NORM_FUSED", "1") != "0"

# GPTQ linears with at least this many input rows dequantise their weight once per call (bf16, N x K, into one
# buffer shared by all layers) and run the bf16 GEMM; fewer rows run the kernel that dequantises each weight
# tile in shared memory (there the int4 weight bytes, not the multiply, bound the call).
GPTQ_DEQUANT_MIN_ROWS = 1024


def _pad_cols(w: torch.Tensor, mult: int = 8) -> torch.Tensor:
    k = w.shape[1]
    kp = (k + mult - 1) // mult * mult
    if kp == k:
        return w
    out = torch.zeros(w.shape[0], kp, dtype=w.dtype)
    out[:, :k] = w
    return out


@dataclass
class Lin:
    """A prepared linear: weight [N, K] (bf16 or e4m3) on the device, optional fp32 per-row scale and bias."""

    w: Optional[torch.Tensor]
    scale: Optional[torch.Tensor]
    bias: Optional[torch.Tensor]
    fp8: bool
    gptq: Optional[dict] = None  # repacked int4 layer (sa3_b200.gptq.repack layout) on the device

    @property
    def n(self):
        return self.gptq["n"] if self.gptq is not None else self.w.shape[0]


class _Workspace:
    """Device buffers and packing tables for one set of sequence lengths (reused across steps and graph replays).

    Sequences are packed back to back as token rows: sequence b occupies stream rows [cu[b], cu[b+1]),
    memory tokens first, then its L_b latents. Every per-row table the kernels take is built here once:
    row_batch (sequence of each row), row_pos (RoPE position), lat_rows (stream row of each latent row)
    and mem_rows (stream rows of the memory tokens).

    With a padding mask (`valid[b]` = sorted indices of sequence b's valid latents) the rows are laid out
    valid-first: rows [0, V) hold every sequence's memory tokens and valid latents back to back (the packed
    tokens of the reference's flash-varlen path, transformer.py:620-651), rows [V, M) the padded latents. The
    self-attention then runs varlen over rows [0, V) with `cu`, the feed-forward runs on rows [0, V) only
    (transformer.py:500-519), and the padded rows keep a zero self-attention output. RoPE positions stay the
    original token positions."""

    def __init__(self, cfg, lengths, Tc: int, dev, fp8: bool, gptq_k: int = 0, local_all: bool = False,
                 split: Optional["_seqsplit.SeqSplit"] = None, kv_all: bool = False, valid=None,
                 stream_dtype: torch.dtype = torch.float16):
        D = cfg.embed_dim
        # a sequence-split rank holds stream tokens [tok_start, tok_end) of each sequence: memory tokens only on
        # rank 0, RoPE at global positions
        nm = cfg.num_memory_tokens if split is None else split.memory_here
        pos0 = 0 if split is None else split.tok_start
        B = len(lengths)
        Ns = [L + nm for L in lengths]
        M = sum(Ns)
        R = sum(lengths)
        nq = 5 if cfg.differential else 3
        self.lengths, self.B, self.M, self.R, self.Tc = tuple(lengths), B, M, R, Tc
        self.max_n = max(Ns)
        self.nm, self.max_pos, self.split = nm, pos0 + max(Ns), split
        # sequences of one length (a CFG pair, a uniform batch): batch(row) = row // N, which lets the norm
        # keep every batch's modulation coefficients in shared memory instead of a per-row table lookup
        self.uniform_n = Ns[0] if all(n == Ns[0] for n in Ns) else 0
        self.lat_off = [int(x) for x in np.concatenate([[0], np.cumsum(lengths)])]
        self.masked = valid is not None
        self.valid = valid
        self.cu_pad = None
        self.max_pad = 0
        if not self.masked:
            cu = np.zeros(B + 1, dtype=np.int64)
            cu[1:] = np.cumsum(Ns)
            row_batch = np.repeat(np.arange(B, dtype=np.int32), Ns)
            row_pos = np.concatenate([pos0 + np.arange(n, dtype=np.int32) for n in Ns])
            lat_rows = np.concatenate([np.arange(cu[b] + nm, cu[b + 1], dtype=np.int32) for b in range(B)])
            mem_rows = (np.concatenate([np.arange(cu[b], cu[b] + nm, dtype=np.int64) for b in range(B)])
                        if nm else None)
            self.V = M
        else:
            if split is not None:
                raise ValueError("a sequence split takes no padding mask")
            nv = [len(v) for v in valid]
            pcount = [n_all - n for n_all, n in zip(lengths, nv)]
            cu = np.zeros(B + 1, dtype=np.int64)
            cu[1:] = np.cumsum([nm + n for n in nv])
            V = int(cu[-1])
            cu_p = np.zeros(B + 1, dtype=np.int64)
            cu_p[1:] = np.cumsum(pcount)
            row_batch = np.empty(M, dtype=np.int32)
            row_pos = np.empty(M, dtype=np.int32)
            lat_rows = np.empty(R, dtype=np.int32)
            mem_rows = []
            for b in range(B):
                vi = np.asarray(valid[b], dtype=np.int64)
                pi = np.setdiff1d(np.arange(lengths[b]), vi)
                r0, r1 = int(cu[b]), int(cu[b + 1])
                row_batch[r0:r1] = b
                row_pos[r0:r0 + nm] = np.arange(nm)
                row_pos[r0 + nm:r1] = nm + vi
                lat_rows[self.lat_off[b] + vi] = r0 + nm + np.arange(len(vi))
                p0, p1 = V + int(cu_p[b]), V + int(cu_p[b + 1])
                row_batch[p0:p1] = b
                row_pos[p0:p1] = nm + pi
                lat_rows[self.lat_off[b] + pi] = p0 + np.arange(len(pi))
                mem_rows.append(np.arange(r0, r0 + nm, dtype=np.int64))
            mem_rows = np.concatenate(mem_rows) if nm else None
            self.V = V
            self.uniform_n = 0
            self.max_n = nm + max(nv)
            self.max_pad = max(pcount)
            self.cu_pad = torch.from_numpy(cu_p.astype(np.int32)).to(dev)
        self.cu_host = cu
        self.cu = torch.from_numpy(cu.astype(np.int32)).to(dev)
        self.cu_ctx = torch.arange(0, (B + 1) * Tc, max(Tc, 1), dtype=torch.int32, device=dev)[:B + 1] if Tc else None
        self.row_batch = torch.from_numpy(row_batch).to(dev)
        self.row_pos = torch.from_numpy(row_pos).to(dev)
        self.lat_rows = torch.from_numpy(lat_rows).to(dev)
        self.mem_rows = torch.from_numpy(mem_rows).to(dev) if nm else None
        bf = torch.bfloat16
        self.h = torch.empty(M, D, device=dev, dtype=stream_dtype)  # residual stream (fp16 or fp32)
        self.a = torch.empty(M, D, device=dev, dtype=torch.float8_e4m3fn if fp8 else bf)
        # 1/rms of each stream row, stored by a norm's max|y| pass and read by its write pass; the grid barrier of
        # the one-launch norm (arrival count, generation)
        self.row_r = torch.empty(M, device=dev, dtype=torch.float32) if fp8 else None
        self.norm_barrier = torch.zeros(2, device=dev, dtype=torch.int32) if fp8 else None
        self.qkv = torch.empty(M, nq * D, device=dev, dtype=bf)
        if split is not None:
            # per sequence [left halo | own rows | right halo] of the q|k|v|q'|k' projection
            if any(n != Ns[0] for n in Ns):
                raise ValueError("a sequence split needs sequences of one length")
            self.halo_e = split.halo_left + Ns[0] + split.halo_right
            self.qkv_ext = torch.empty(B * self.halo_e, nq * D, device=dev, dtype=bf)
        # self-attention output; with a padding mask its padded rows stay zero (no attention writes them) and
        # cross-attention writes a buffer of its own
        self.o = torch.zeros(M, D, device=dev, dtype=bf) if self.masked else torch.empty(M, D, device=dev, dtype=bf)
        self.ox = torch.empty(M, D, device=dev, dtype=bf) if self.masked else self.o
        self.o8 = torch.empty(M, D, device=dev, dtype=torch.float8_e4m3fn) if fp8 else None
        self.qx = torch.empty(M, (2 if cfg.differential else 1) * D, device=dev, dtype=bf)
        self.kv = torch.empty(max(B * Tc, 1), (3 if cfg.differential else 2) * D, device=dev, dtype=bf)
        # every block's cross-attention K/V, computed once per forward
        self.kv_all = torch.empty(max(B * Tc, 1), cfg.depth * (3 if cfg.differential else 2) * D, device=dev,
                                  dtype=bf) if Tc and kv_all else None
        self.u = torch.empty(M, cfg.ff_inner, device=dev, dtype=bf)
        self.u8 = torch.empty(M, cfg.ff_inner, device=dev, dtype=torch.float8_e4m3fn) if fp8 else None
        # The local conditioning (transformer.py:978-994) runs over all M stream rows in stream order: its input
        # rows are the latent rows' conditioning with zero rows at the memory tokens, and its output is added in
        # place with a per-row gate factor of exactly 1 on latent rows and 0 on memory tokens (stream_kind), so
        # the memory tokens get no conditioning, as the reference's left padding gives them (:77-88).
        self.t1 = torch.empty(M, D, device=dev, dtype=bf)
        # every block's first local-conditioning layer, computed once per forward (within a byte budget)
        self.t1_all = None
        if local_all and M * cfg.depth * D * 2 <= _LOCAL_ALL_MAX_BYTES:
            self.t1_all = torch.empty(M, cfg.depth * D, device=dev, dtype=bf)
        self.loc = torch.zeros(R, 264, device=dev, dtype=bf)  # latent order, as the caller passes it
        self.loc_s = torch.zeros(M, 264, device=dev, dtype=bf)  # stream order; memory-token rows stay zero
        self.lat_rows_l = self.lat_rows.long()
        kind = torch.zeros(M, dtype=torch.int32)
        if mem_rows is not None:
            kind[torch.from_numpy(mem_rows).long()] = 1
        self.stream_kind = kind.to(dev)
        self.xin = torch.empty(R, cfg.io_channels, device=dev, dtype=bf)
        self.hb = torch.empty(R, D, device=dev, dtype=bf)  # bf16 copy of the latent rows for project_out
        self.out = torch.empty(R, cfg.io_channels, device=dev, dtype=torch.float32)
        self.ctx = torch.empty(max(B * Tc, 1), D, device=dev, dtype=bf)
        self.ctx8 = torch.empty(max(B * Tc, 1), D, device=dev, dtype=torch.float8_e4m3fn) if fp8 else None
        self.nslots = 8 * cfg.depth + 8
        self.amax = torch.zeros(self.nslots, device=dev, dtype=torch.float32)
        self.scale = torch.zeros(self.nslots, device=dev, dtype=torch.float32)
        self.small = torch.empty(B, 8 * D, device=dev, dtype=bf)
        # act-order gather buffer of the GPTQ path (inputs of every int4 linear)
        self.xperm = torch.empty(max(M, B * Tc), gptq_k, device=dev, dtype=bf) if gptq_k else None


class DiTEngine:
    def __init__(self, module, mode: str = "bf16", gptq_layers: Optional[dict] = None, device="cuda",
                 stream_dtype: torch.dtype = torch.float16):
        if mode not in ("bf16", "fp8", "gptq"):
            raise ValueError(mode)
        if stream_dtype not in (torch.float16, torch.float32):
            raise ValueError(f"residual stream dtype {stream_dtype}: fp16 or fp32")
        self.stream_dtype = stream_dtype
        if not torch.cuda.is_available():
            raise RuntimeError("DiTEngine needs a CUDA device (no CPU path)")
        _lib.load()
        self.cfg = cfg = module.cfg
        self.mode = mode
        self.fp8 = mode == "fp8"
        self.dev = torch.device(device)
        if cfg.head_dim != 64:
            raise NotImplementedError("head_dim must be 64")
        sd = {k: v.detach().float().cpu() for k, v in module.state_dict().items()}
        self.gptq_layers = gptq_layers or {}
        if mode == "gptq" and not self.gptq_layers:
            raise ValueError("mode 'gptq' needs gptq_layers (name -> GPTQ tensors or a repacked layer)")
        self.lin: Dict[str, Lin] = {}
        for name in sorted({k[:-len(".weight")] for k in sd if k.endswith(".weight")}):
            if name in ("preprocess_conv", "postprocess_conv", "transformer.project_in", "transformer.project_out"):
                continue
            quantized = self.fp8 and any(name.endswith(s) for s in QUANT_SUFFIXES)
            self.lin[name] = self._prep(name, sd[name + ".weight"], sd.get(name + ".bias"), quantized)
        D = cfg.embed_dim
        eye = torch.eye(cfg.io_channels)
        w_in = sd["transformer.project_in.weight"] @ (eye + sd["preprocess_conv.weight"][:, :, 0])
        w_out = (eye + sd["postprocess_conv.weight"][:, :, 0]) @ sd["transformer.project_out.weight"]
        self.lin["project_in"] = Lin(w_in.to(self.dev, torch.bfloat16).contiguous(), None, None, False)
        self.lin["project_out"] = Lin(w_out.to(self.dev, torch.bfloat16).contiguous(), None, None, False)
        self.memory = sd["transformer.memory_tokens"].to(self.dev, stream_dtype) if cfg.num_memory_tokens else None
        self.sst = torch.stack([sd[f"transformer.layers.{i}.to_scale_shift_gate"] for i in range(cfg.depth)]).to(
            self.dev)
        self.gam = {k: v.to(self.dev).contiguous() for k, v in sd.items() if k.endswith("gamma")}
        # gate rows of the local-conditioning add: sigmoid(1 - g) is exactly 1 for g = -inf (latent rows) and
        # exactly 0 for g = +inf (memory tokens)
        self.loc_gate = torch.tensor([-math.inf, math.inf], device=self.dev).repeat_interleave(
            cfg.embed_dim).view(2, cfg.embed_dim).contiguous()
        self.rope = None
        self.ws: Optional[_Workspace] = None
        ramp = torch.linspace(0, 1, cfg.timestep_features_dim // 2, dtype=torch.float32)
        self.t_freqs = torch.exp(ramp * (math.log(10000.0) - math.log(0.5)) + math.log(0.5)).to(self.dev)
        self.gptq_k = max([ln.gptq["k"] for ln in self.lin.values() if ln.gptq is not None], default=0)
        # transient dense weight of the large-batch GPTQ path (the largest layer: 38 MB for the medium GLU.proj)
        nk = max([ln.gptq["n"] * ln.gptq["k"] for ln in self.lin.values() if ln.gptq is not None], default=0)
        self.wdq = torch.empty(nk, device=self.dev, dtype=torch.bfloat16) if nk else None
        self._prep_kv_all()
        self._prep_local_all()

    def _prep_local_all(self):
        """The first local-conditioning layer of all blocks as one linear: its input (the padded local
        conditioning rows) is the same for every block, so one GEMM per forward replaces one per block."""
        L = self.cfg.depth
        names = [f"transformer.layers.{i}.to_local_embed.0" for i in range(L)]
        self.loc1_all = None
        if not all(n in self.lin and self.lin[n].gptq is None and not self.lin[n].fp8 for n in names):
            return
        lins = [self.lin[n] for n in names]
        if any(ln.w.shape[0] != self.cfg.embed_dim for ln in lins):
            return
        w = torch.cat([ln.w for ln in lins]).contiguous()
        bias = None
        if any(ln.bias is not None for ln in lins):
            bias = torch.cat([ln.bias if ln.bias is not None else torch.zeros(ln.w.shape[0], device=self.dev)
                              for ln in lins]).contiguous()
        self.loc1_all = Lin(w, None, bias, False)

    def _prep_kv_all(self):
        """The cross-attention K/V projections of all blocks as one linear (the context is the same for every
        block, so one GEMM per step replaces one small GEMM per block). Output columns are grouped
        [k_0 | k'_0 | ... | k_{L-1} | k'_{L-1} | v_0 | ... | v_{L-1}] (k' only when differential); the k groups
        are k-normalised with their block's gamma from a table, the v groups are stored as computed."""
        cfg = self.cfg
        D, L = cfg.embed_dim, cfg.depth
        names = [f"transformer.layers.{i}.cross_attn.to_kv" for i in range(L)]
        self.kv_all = None
        gnames = [f"transformer.layers.{i}.cross_attn.k_norm.gamma" for i in range(L)]
        if not all(n in self.lin and self.lin[n].gptq is None for n in names) or not all(g in self.gam for g in gnames):
            return
        lins = [self.lin[n] for n in names]
        nk = 2 if cfg.differential else 1
        order = [(i, j) for i in range(L) for j in range(nk)] + [(i, nk) for i in range(L)]
        w = torch.cat([lins[i].w[j * D:(j + 1) * D] for i, j in order]).contiguous()
        scale = torch.cat([lins[i].scale[j * D:(j + 1) * D] for i, j in order]).contiguous() if lins[0].fp8 else None
        bias = None
        if any(ln.bias is not None for ln in lins):
            bias = torch.cat([(lins[i].bias[j * D:(j + 1) * D] if lins[i].bias is not None
                               else torch.zeros(D, device=self.dev)) for i, j in order]).contiguous()
        gk = [self.gam[g] for g in gnames]
        self.kv_gamma = torch.stack([gk[i] for i in range(L) for _ in range(nk)]).float().contiguous()
        self.kv_all = Lin(w, scale, bias, lins[0].fp8)
        self.kv_nk = nk

    # ------------------------------------------------------------------ prep
    def _prep(self, name, w, b, quantized: bool) -> Lin:
        if self.mode == "gptq" and name in self.gptq_layers:
            packed = self.gptq_layers[name]
            if not isinstance(packed, dict):  # raw GPTQ tensors (qweight, qzeros, scales, g_idx)
                packed = _gptq.repack(*packed)
            packed = _gptq.to_device(packed, self.dev)
            if name.endswith("ff.ff.0.proj"):
                idx = swiglu_interleave_index(packed["n"])
                packed = _gptq.reorder_rows(packed, idx)
                b = None if b is None else b[idx]
            bias = None if b is None else b.to(self.dev, torch.float32).contiguous()
            return Lin(None, None, bias, False, packed)
        if name.endswith("ff.ff.0.proj"):
            w, b = interleave_swiglu_rows(w, b)
        w = _pad_cols(w)
        bias = None if b is None else b.to(self.dev, torch.float32).contiguous()
        if quantized:
            wq, s = quantize_weight_e4m3(w)
            return Lin(wq.to(self.dev).contiguous(), s.to(self.dev), bias, True)
        return Lin(w.to(self.dev, torch.bfloat16).contiguous(), None, bias, False)

    def _workspace(self, lengths, Tc, split=None, valid=None) -> _Workspace:
        ws = self.ws
        vkey = None if valid is None else tuple(np.asarray(v, dtype=np.int64).tobytes() for v in valid)
        if ws is None or (ws.lengths, ws.Tc, ws.split, ws.valid_key) != (tuple(lengths), Tc, split, vkey):
            self.ws = ws = None
            self.ws = ws = _Workspace(self.cfg, lengths, Tc, self.dev, self.fp8, self.gptq_k,
                                      local_all=self.loc1_all is not None, split=split,
                                      kv_all=self.kv_all is not None, valid=valid, stream_dtype=self.stream_dtype)
            ws.valid_key = vkey
            if split is not None and split.world > 1 and self.fp8:
                # collective set-up of the peer-memory amax exchange (every rank builds its workspace here)
                _seqsplit.prepare_peer_max(split.group)
        if self.rope is None or self.rope.shape[0] < ws.max_pos:
            self.rope = ops.rope_table(ws.max_pos, 32, device=self.dev)
        return ws

    # ------------------------------------------------------------------ helpers
    def _gemm(self, x, lin: Lin, out=None, x_scale=None, **kw):
        if lin.gptq is not None:
            g = lin.gptq
            if x.shape[0] >= GPTQ_DEQUANT_MIN_ROWS and "inv_perm" in g:
                # many rows: dequantise the int4 weight once, in the original channel order, and run the bf16
                # GEMM on the unpermuted activations (no act-order gather, no per-tile dequantisation)
                w = ops.gptq_dequant_orig(g["qw"], g["sz"], g["inv_perm"], g["n"], g["k"], g["group_size"],
                                          out=self.wdq[:g["n"] * g["k"]].view(g["n"], g["k"]))
                return ops.gemm(x, w, out, bias=lin.bias, **kw)
            xp = ops.permute_cols(x, g["perm"], self.ws.xperm[:x.shape[0], :g["k"]])
            return ops.gptq_gemm(xp, g["qw"], g["sz"], g["n"], out, group_size=g["group_size"], bias=lin.bias, **kw)
        if lin.fp8 and x.dtype != torch.float8_e4m3fn:
            raise RuntimeError("fp8 linear needs a quantized activation")
        return ops.gemm(x, lin.w, out, a_scale=x_scale if lin.fp8 else None, b_scale=lin.scale, bias=lin.bias, **kw)

    def _norm_to_a(self, ws, x, gamma, slot, mod=None, scale_off=0, shift_off=0):
        """RMSNorm(+modulate) of the first x.shape[0] stream rows into ws.a; FP8: two passes (amax, quantize)."""
        cfg = self.cfg
        rows = x.shape[0]
        a = ws.a[:rows]
        if ws.uniform_n:
            kw = dict(mod=mod, scale_off=scale_off, shift_off=shift_off, rows_per_batch=ws.uniform_n)
        else:
            kw = dict(mod=mod, scale_off=scale_off, shift_off=shift_off, row_batch=ws.row_batch[:rows])
        if self.fp8:
            am = ws.amax[slot:slot + 1]
            sc = ws.scale[slot:slot + 1]
            rr = ws.row_r[:rows]
            if _NORM_ONE_LAUNCH and (ws.split is None or ws.split.world == 1):
                # both passes in one launch where the kernel serves the shape
                ops.rmsnorm_quant_fused(x, gamma, cfg.norm_eps, out=a, amax=am, row_r=rr, barrier=ws.norm_barrier,
                                        scale_out=sc, **kw)
                return a, sc
            ops.rmsnorm_modulate(x, gamma, cfg.norm_eps, amax_only=am, row_r=rr, **kw)
            self._sync_amax(ws, slot)
            ops.rmsnorm_modulate(x, gamma, cfg.norm_eps, out=a, quant_amax=am, scale_out=sc, row_r=rr, **kw)
            return a, sc
        ops.rmsnorm_modulate(x, gamma, cfg.norm_eps, out=a, **kw)
        return a, None

    @staticmethod
    def _sync_amax(ws, slot):
        """Sequence split: the per-tensor activation scale spans the whole sequence, as in the unsplit step, so
        each rank's max|x| at a quantisation point is max-reduced over the split's ranks before it is used."""
        sp = ws.split
        if sp is not None and sp.world > 1:
            _seqsplit.all_reduce_max(ws.amax[slot:slot + 1], sp.group)

    def _quant(self, ws, x, out8, slot):
        """FP8: quantize x (whose amax is already in slot) into out8; bf16: pass x through."""
        if not self.fp8:
            return x, None
        self._sync_amax(ws, slot)
        sc = ws.scale[slot:slot + 1]
        ops.quantize_e4m3(x, ws.amax[slot:slot + 1], out=out8, scale_out=sc)
        return out8, sc

    def _split_self_attention(self, ws, a, asc, lin, groups, rope, o, amax_out, wl, wr):
        """Self-attention of a sequence-split rank: the q|k|v|q'|k' projection of each sequence lands between
        its halo rows, the boundary rows are exchanged with the neighbouring ranks, and the queries of the
        own rows attend over [left halo | own | right halo] with the window re-centred: the interior queries
        while the exchange is in flight, the queries next to a neighbour after it."""
        cfg, sp = self.cfg, ws.split
        if (sp.wl, sp.wr) != (wl, wr):
            raise ValueError(f"split made for window {(sp.wl, sp.wr)}, the model attends over {(wl, wr)}")
        D, H, n, e, hl = cfg.embed_dim, cfg.num_heads, ws.uniform_n, ws.halo_e, sp.halo_left
        ext = ws.qkv_ext
        for b in range(ws.B):
            self._gemm(a[b * n:(b + 1) * n], lin, ext[b * e + hl:b * e + hl + n], x_scale=asc, kind=_lib.EPI_QK_NORM,
                       qk=dict(gammas=groups, group_width=D, rope=rope, eps=cfg.qk_norm_eps, cos_sin=self.rope,
                               row_pos=ws.row_pos[b * n:(b + 1) * n]))
        # the halo transfers run while the interior queries (windows inside the own rows) are attended
        reqs = _seqsplit.exchange_halos(ext, ws.B, n, sp, wait=False)
        interior, edges = _seqsplit.attention_views(n, sp)

        def attend(views):
            for b in range(ws.B):
                blk = ext[b * e:(b + 1) * e]
                for q0, q1, k0, k1, win in views:
                    q, k = blk[hl + q0:hl + q1], blk[k0:k1]
                    kw = dict(heads=H, window=win, out=o[b * n + q0:b * n + q1], amax_out=amax_out, batch=1,
                              max_seqlen_q=q1 - q0, max_seqlen_k=k1 - k0)
                    if cfg.differential:
                        ops.attention(q[:, 0:D], k[:, D:2 * D], k[:, 2 * D:3 * D], q2=q[:, 3 * D:4 * D],
                                      k2=k[:, 4 * D:5 * D], **kw)
                    else:
                        ops.attention(q[:, 0:D], k[:, D:2 * D], k[:, 2 * D:3 * D], **kw)

        attend(interior)
        for req in reqs:
            req.wait()
        attend(edges)

    # ------------------------------------------------------------------ forward
    @torch.no_grad()
    def forward_split(self, x, t, split, cross_attn_cond=None, global_embed=None, local_add_cond=None,
                      cfg_scale: float = 1.0, apg_scale: float = 1.0):
        """DiffusionTransformer.forward on this rank's share of one long sequence (sa3_b200.seqsplit): x and
        local_add_cond hold the latent columns [split.lat_start, split.lat_end); every rank of split.group calls
        this with the same t / conditioning. Returns this rank's columns of the velocity."""
        dev = self.dev
        x = x.to(dev)
        t = t.to(dev, torch.float32)
        if cfg_scale != 1.0 and cross_attn_cond is not None:
            cc = cross_attn_cond.to(dev)
            bg = torch.cat([global_embed, global_embed]).to(dev) if global_embed is not None else None
            bl = torch.cat([local_add_cond, local_add_cond]).to(dev) if local_add_cond is not None else None
            out = self.inner_split(torch.cat([x, x]), torch.cat([t, t]), split, torch.cat([cc, torch.zeros_like(cc)]),
                                   bg, bl)
            return _seqsplit.cfg_combine_split(x, t, out, cfg_scale, apg_scale, split.group)
        return self.inner_split(x, t, split, cross_attn_cond, global_embed, local_add_cond)

    @torch.no_grad()
    def inner_split(self, x, t, split, cross_attn_cond=None, global_embed=None, local_add_cond=None):
        """`inner` on a sequence-split rank: x [B, C, lat_end - lat_start] (B sequences of one length, all split
        the same way); returns fp32 [B, C, lat_end - lat_start]."""
        B, C, L = x.shape
        if L != split.lat_end - split.lat_start:
            raise ValueError(f"rank {split.rank} holds {split.lat_end - split.lat_start} latents, got {L}")
        Tc = cross_attn_cond.shape[1] if cross_attn_cond is not None else 0
        ws = self._workspace([L] * B, Tc, split)
        ws.xin.view(B, L, C).copy_(x.transpose(1, 2))
        if local_add_cond is not None and self.cfg.local_add_cond_dim > 0:
            ws.loc.view(B, L, -1)[:, :, :self.cfg.local_add_cond_dim].copy_(local_add_cond.transpose(1, 2))
        self._trunk(ws, t, cross_attn_cond, global_embed, local_add_cond is not None)
        return ws.out.view(B, L, C).transpose(1, 2)

    @torch.no_grad()
    def forward(self, x, t, cross_attn_cond=None, global_embed=None, local_add_cond=None, cfg_scale: float = 1.0,
                apg_scale: float = 1.0, padding_mask=None):
        """DiffusionTransformer.forward for the rf_denoiser objective (dit.py:345-643). padding_mask [B, L] bool
        (True = valid latent) selects the reference's varlen semantics; both CFG halves share it (dit.py:549-550)
        and the APG projection is restricted to valid positions (dit.py:311-343)."""
        dev = self.dev
        x = x.to(dev)
        t = t.to(dev, torch.float32)
        if cfg_scale != 1.0 and cross_attn_cond is not None:
            bx = torch.cat([x, x])
            bt = torch.cat([t, t])
            cc = cross_attn_cond.to(dev)
            bc = torch.cat([cc, torch.zeros_like(cc)])
            bg = torch.cat([global_embed, global_embed]).to(dev) if global_embed is not None else None
            bl = torch.cat([local_add_cond, local_add_cond]).to(dev) if local_add_cond is not None else None
            bm = torch.cat([padding_mask, padding_mask]) if padding_mask is not None else None
            out = self.inner(bx, bt, bc, bg, bl, padding_mask=bm)
            return self.cfg_combine(x, t, out, cfg_scale, apg_scale, padding_mask)
        return self.inner(x, t, cross_attn_cond, global_embed, local_add_cond, padding_mask=padding_mask)

    def graphed(self, x, t, cross_attn_cond=None, global_embed=None, local_add_cond=None, cfg_scale: float = 1.0,
                apg_scale: float = 1.0, padding_mask=None) -> "GraphedStep":
        """Capture one forward at these shapes into a CUDA graph (inputs are copied into static buffers). The
        padding mask is part of what is captured (it fixes the row layout); replays use the same mask."""
        return GraphedStep(self, (x, t, cross_attn_cond, global_embed, local_add_cond), cfg_scale, apg_scale,
                           padding_mask)

    def cfg_combine(self, x, t, out, cfg_scale, apg_scale, padding_mask=None):
        """CFG + APG for rf_denoiser (dit.py:571-625; apg_project dit.py:311-343), fp32. With a padding mask the
        projection direction is cond_den on valid positions (norm floored at 1e-8) and the orthogonal part is
        zero on padded positions."""
        x = x.float()
        cond_out, uncond_out = out.float().chunk(2)
        sigma = t.float()[:, None, None]
        cond_den = x - cond_out * sigma
        diff = (uncond_out - cond_out) * sigma  # cond_den - uncond_den
        if apg_scale == 0.0:
            cfg_diff = diff
        elif padding_mask is None:
            v1 = cond_den / cond_den.flatten(1).norm(dim=1).clamp_min(1e-12)[:, None, None]
            par = (diff * v1).sum(dim=(1, 2), keepdim=True) * v1
            orth = diff - par
            cfg_diff = orth if apg_scale == 1.0 else apg_scale * orth + (1 - apg_scale) * diff
        else:
            mask = padding_mask.to(x.device)[:, None, :].float()
            v1 = cond_den * mask
            v1 = v1 / v1.flatten(1).norm(dim=1).clamp_min(1e-8)[:, None, None]
            orth = (diff - (diff * v1).sum(dim=(1, 2), keepdim=True) * v1) * mask
            cfg_diff = orth if apg_scale == 1.0 else apg_scale * orth + (1 - apg_scale) * diff
        cfg_den = cond_den + (cfg_scale - 1) * cfg_diff
        return (x - cfg_den) / sigma

    def _valid_latents(self, padding_mask, B: int, L: int):
        """Host-side list of each sequence's valid latent indices, or None when every latent is valid (the
        unmasked path computes the same thing). Reading the mask is the one host sync the mask costs, as the
        reference's own varlen metadata does (transformer.py:57-58). Under CUDA-graph capture the mask cannot
        be read: the warm-up forward that precedes every capture has laid out the workspace for it."""
        if padding_mask is None:
            return None
        if torch.cuda.is_current_stream_capturing():
            if self.ws is None or self.ws.lengths != tuple([L] * B):
                raise RuntimeError("padding_mask under graph capture needs a warm-up forward with the same mask")
            return self.ws.valid
        pm = padding_mask.detach().to("cpu", torch.bool)
        if tuple(pm.shape) != (B, L):
            raise ValueError(f"padding_mask must be [{B}, {L}], got {tuple(pm.shape)}")
        if bool(pm.all()):
            return None
        return [np.nonzero(pm[b].numpy())[0] for b in range(B)]

    @torch.no_grad()
    def inner(self, x, t, cross_attn_cond=None, global_embed=None, local_add_cond=None, padding_mask=None):
        """DiffusionTransformer._forward + ContinuousTransformer.forward on the kernels for B sequences of one
        length; returns fp32 [B, C, L]. padding_mask [B, L] bool (True = valid latent) as in
        ContinuousTransformer.forward (transformer.py:1213-1232)."""
        B, C, L = x.shape
        Tc = cross_attn_cond.shape[1] if cross_attn_cond is not None else 0
        ws = self._workspace([L] * B, Tc, valid=self._valid_latents(padding_mask, B, L))
        ws.xin.view(B, L, C).copy_(x.transpose(1, 2))
        if local_add_cond is not None and self.cfg.local_add_cond_dim > 0:
            ws.loc.view(B, L, -1)[:, :, :self.cfg.local_add_cond_dim].copy_(local_add_cond.transpose(1, 2))
        self._trunk(ws, t, cross_attn_cond, global_embed, local_add_cond is not None)
        return ws.out.view(B, L, C).transpose(1, 2)

    @torch.no_grad()
    def inner_varlen(self, xs, t, cross_attn_cond=None, global_embed=None, local_add_conds=None):
        """Variable-length batch: xs = list of [C, L_b] latents (local_add_conds likewise [257, L_b]); t [B],
        cross_attn_cond [B, Tc, 768], global_embed [B, 768]. The sequences are packed back to back (no
        padding); returns a list of fp32 [C, L_b]."""
        lengths = [int(x.shape[-1]) for x in xs]
        Tc = cross_attn_cond.shape[1] if cross_attn_cond is not None else 0
        ws = self._workspace(lengths, Tc)
        dev = self.dev
        for b, x in enumerate(xs):
            ws.xin[ws.lat_off[b]:ws.lat_off[b + 1]].copy_(x.to(dev).transpose(0, 1))
        has_local = local_add_conds is not None and self.cfg.local_add_cond_dim > 0
        if has_local:
            for b, lc in enumerate(local_add_conds):
                ws.loc[ws.lat_off[b]:ws.lat_off[b + 1], :self.cfg.local_add_cond_dim].copy_(lc.transpose(0, 1))
        self._trunk(ws, t.to(dev), None if cross_attn_cond is None else cross_attn_cond.to(dev),
                    None if global_embed is None else global_embed.to(dev), has_local)
        return [ws.out[ws.lat_off[b]:ws.lat_off[b + 1]].transpose(0, 1) for b in range(len(xs))]

    @torch.no_grad()
    def forward_varlen(self, xs, t, cross_attn_cond, global_embed=None, local_add_conds=None, cfg_scale: float = 1.0,
                       apg_scale: float = 1.0):
        """DiffusionTransformer.forward over prompts of different lengths: each prompt's CFG pair runs in one
        packed batch (cond halves first, then the unconditional halves), then the per-prompt CFG/APG combine."""
        P = len(xs)
        dev = self.dev
        t = t.to(dev, torch.float32)
        if cfg_scale == 1.0:
            return self.inner_varlen(xs, t, cross_attn_cond, global_embed, local_add_conds)
        cc = cross_attn_cond.to(dev)
        outs = self.inner_varlen(
            list(xs) + list(xs), torch.cat([t, t]), torch.cat([cc, torch.zeros_like(cc)]),
            None if global_embed is None else torch.cat([global_embed, global_embed]).to(dev),
            None if local_add_conds is None else list(local_add_conds) + list(local_add_conds))
        res = []
        for i in range(P):
            pair = torch.stack([outs[i], outs[P + i]])
            res.append(self.cfg_combine(xs[i].to(dev)[None], t[i:i + 1], pair, cfg_scale, apg_scale)[0])
        return res

    def _trunk(self, ws: _Workspace, t, cross_attn_cond, global_embed, has_local: bool):
        """The trunk on packed sequences: reads ws.xin / ws.loc, writes ws.out (fp32 [R, C])."""
        cfg = self.cfg
        D = cfg.embed_dim
        B, Tc = ws.B, ws.Tc
        nm = ws.nm
        ln = self.lin
        ws.amax.zero_()

        # ---- conditioning prologue (dit.py:197-262, transformer.py:1210-1211)
        tf = t.float()[:, None] * self.t_freqs[None, :] * (2 * math.pi)
        feats = torch.cat([torch.cos(tf), torch.sin(tf)], dim=-1).to(torch.bfloat16)
        sm = ws.small
        temb1 = self._gemm(feats, ln["to_timestep_embed.0"], sm[:, 0:D], kind=_lib.EPI_SILU)
        temb = self._gemm(temb1, ln["to_timestep_embed.2"], sm[:, D:2 * D])
        if global_embed is not None:
            ge = global_embed.to(torch.bfloat16).contiguous()
            g1 = self._gemm(ge, ln["to_global_embed.0"], sm[:, 2 * D:3 * D], kind=_lib.EPI_SILU)
            g = self._gemm(g1, ln["to_global_embed.2"], sm[:, 3 * D:4 * D], kind=_lib.EPI_RESIDUAL, residual=temb)
        else:
            g = temb
        e1 = self._gemm(g, ln["transformer.global_cond_embedder.0"], sm[:, 4 * D:5 * D], kind=_lib.EPI_SILU)
        g6 = self._gemm(e1, ln["transformer.global_cond_embedder.2"])  # [B, 6D]
        ss = (self.sst[:, None, :] + g6.float()[None]).contiguous()    # [depth, B, 6D] fp32

        ctx = None
        if cross_attn_cond is not None:
            cc = cross_attn_cond.reshape(B * Tc, -1).to(torch.bfloat16).contiguous()
            c1 = self._gemm(cc, ln["to_cond_embed.0"], kind=_lib.EPI_SILU)
            ctx = self._gemm(c1, ln["to_cond_embed.2"], ws.ctx)
        ctx_a, ctx_s = ctx, None
        if ctx is not None and self.fp8:
            slot = 8 * cfg.depth
            ops.absmax(ctx, ws.amax[slot:slot + 1])
            ctx_a, ctx_s = self._quant(ws, ctx, ws.ctx8, slot)
        t1_all = None
        if has_local:
            ws.loc_s.index_copy_(0, ws.lat_rows_l, ws.loc)  # latent rows into stream order
        if has_local and ws.t1_all is not None:
            # every block's SiLU(W1 c + b1) of the local conditioning in one GEMM
            t1_all = self._gemm(ws.loc_s, self.loc1_all, ws.t1_all, kind=_lib.EPI_SILU)
        kv_all = None
        if ctx is not None and self.kv_all is not None:
            # every block's cross-attention K/V (with k-norm) in one GEMM
            kv_all = self._gemm(ctx_a, self.kv_all, ws.kv_all, x_scale=ctx_s, kind=_lib.EPI_QK_NORM,
                                qk=dict(gamma_table=self.kv_gamma, group_width=D, eps=cfg.qk_norm_eps))

        # ---- trunk input: project_in (preprocess conv folded) into each sequence's latent rows
        h = ws.h
        self._gemm(ws.xin, ln["project_in"], h, out_row_map=ws.lat_rows)
        if nm:
            h.index_copy_(0, ws.mem_rows, self.memory.repeat(B, 1))

        wl, wr = cfg.sliding_window if cfg.sliding_window is not None else (-1, -1)
        diff = cfg.differential
        qkv, o, qx, kv = ws.qkv, ws.o, ws.qx, ws.kv
        H = cfg.num_heads
        seq = dict(cu_seqlens_q=ws.cu, cu_seqlens_k=ws.cu, max_seqlen_q=ws.max_n, max_seqlen_k=ws.max_n)
        xseq = dict(cu_seqlens_q=ws.cu, cu_seqlens_k=ws.cu_ctx, max_seqlen_q=ws.max_n, max_seqlen_k=Tc)
        rb = ws.row_batch
        for i in range(cfg.depth):
            p = f"transformer.layers.{i}."
            ssi = ss[i]
            s0 = 8 * i
            # -- self-attention with adaLN (transformer.py:1018-1029)
            a, asc = self._norm_to_a(ws, h, self.gam[p + "pre_norm.gamma"], s0, ssi, 0, D)
            gq, gk = self.gam[p + "self_attn.q_norm.gamma"], self.gam[p + "self_attn.k_norm.gamma"]
            # to_qkv with qk RMSNorm + RoPE fused into the epilogue (groups q | k | v | q_diff | k_diff)
            groups = [gq, gk, None, gq, gk] if diff else [gq, gk, None]
            rope = [True, True, False, True, True] if diff else [True, True, False]
            am1 = ws.amax[s0 + 1:s0 + 2] if self.fp8 else None
            if ws.split is not None:
                self._split_self_attention(ws, a, asc, ln[p + "self_attn.to_qkv"], groups, rope, o, am1, wl, wr)
            else:
                self._gemm(a, ln[p + "self_attn.to_qkv"], qkv, x_scale=asc, kind=_lib.EPI_QK_NORM,
                           qk=dict(gammas=groups, group_width=D, rope=rope, eps=cfg.qk_norm_eps, cos_sin=self.rope,
                                   row_pos=ws.row_pos))
                # varlen over the sequences' rows; with a padding mask only the valid rows [0, V) attend and
                # are attended, and the padded rows' output stays zero (pad_input, transformer.py:650)
                sq = qkv[:ws.V]
                if diff:
                    ops.attention(sq[:, 0:D], sq[:, D:2 * D], sq[:, 2 * D:3 * D], q2=sq[:, 3 * D:4 * D],
                                  k2=sq[:, 4 * D:5 * D], heads=H, window=(wl, wr), out=o[:ws.V], amax_out=am1, **seq)
                else:
                    ops.attention(sq[:, 0:D], sq[:, D:2 * D], sq[:, 2 * D:3 * D], heads=H, window=(wl, wr),
                                  out=o[:ws.V], amax_out=am1, **seq)
            oa, osc = self._quant(ws, o, ws.o8, s0 + 1)
            self._gemm(oa, ln[p + "self_attn.to_out"], h, x_scale=osc, kind=_lib.EPI_GATED_RESIDUAL, residual=h,
                       gate=ssi[:, 2 * D:3 * D], row_batch=rb)
            # -- cross-attention (transformer.py:1031-1035), no adaLN, no RoPE
            if ctx is not None and (p + "cross_attn.to_q") in ln:
                c, csc = self._norm_to_a(ws, h, self.gam[p + "cross_attend_norm.gamma"], s0 + 2)
                gq, gk = self.gam[p + "cross_attn.q_norm.gamma"], self.gam[p + "cross_attn.k_norm.gamma"]
                # to_q / to_kv with the qk RMSNorm fused into the epilogue (no RoPE on cross-attention)
                self._gemm(c, ln[p + "cross_attn.to_q"], qx, x_scale=csc, kind=_lib.EPI_QK_NORM,
                           qk=dict(gammas=[gq, gq] if diff else [gq], group_width=D, eps=cfg.qk_norm_eps))
                if kv_all is not None:
                    nk = self.kv_nk
                    kc = [kv_all[:, (i * nk + j) * D:(i * nk + j + 1) * D] for j in range(nk)]
                    vc = kv_all[:, (cfg.depth * nk + i) * D:(cfg.depth * nk + i + 1) * D]
                else:
                    self._gemm(ctx_a, ln[p + "cross_attn.to_kv"], kv, x_scale=ctx_s, kind=_lib.EPI_QK_NORM,
                               qk=dict(gammas=[gk, gk, None] if diff else [gk, None], group_width=D,
                                       eps=cfg.qk_norm_eps))
                    kc = [kv[:, 0:D], kv[:, D:2 * D]] if diff else [kv[:, 0:D]]
                    vc = kv[:, 2 * D:3 * D] if diff else kv[:, D:2 * D]
                am = ws.amax[s0 + 3:s0 + 4] if self.fp8 else None
                ox = ws.ox
                # with a padding mask the rows of a sequence sit in two segments (valid rows, then padded rows);
                # both attend over the whole context, as the reference's unmasked cross-attention does
                segs = [(0, ws.V, xseq)]
                if ws.V < ws.M:
                    segs.append((ws.V, ws.M, dict(xseq, cu_seqlens_q=ws.cu_pad, max_seqlen_q=ws.max_pad)))
                for r0, r1, kw in segs:
                    if diff:
                        ops.attention(qx[r0:r1, 0:D], kc[0], vc, q2=qx[r0:r1, D:2 * D], k2=kc[1], heads=H,
                                      out=ox[r0:r1], amax_out=am, **kw)
                    else:
                        ops.attention(qx[r0:r1], kc[0], vc, heads=H, out=ox[r0:r1], amax_out=am, **kw)
                oa, osc = self._quant(ws, ox, ws.o8, s0 + 3)
                self._gemm(oa, ln[p + "cross_attn.to_out"], h, x_scale=osc, kind=_lib.EPI_RESIDUAL, residual=h)
            # -- local additive conditioning, left-padded over the memory tokens (transformer.py:978-994, 77-88)
            if has_local and (p + "to_local_embed.0") in ln:
                if t1_all is not None:
                    t1 = t1_all[:, i * D:(i + 1) * D]
                else:
                    t1 = self._gemm(ws.loc_s, ln[p + "to_local_embed.0"], ws.t1, kind=_lib.EPI_SILU)
                self._gemm(t1, ln[p + "to_local_embed.2"], h, kind=_lib.EPI_GATED_RESIDUAL, residual=h,
                           gate=self.loc_gate, row_batch=ws.stream_kind)
            # -- feed-forward with adaLN (transformer.py:1042-1049); with a padding mask only the valid rows
            # [0, V) (transformer.py:500-519: padded rows get a zero FF branch, so they are left as they are)
            V = ws.V
            hv = h[:V]
            f, fsc = self._norm_to_a(ws, hv, self.gam[p + "ff_norm.gamma"], s0 + 4, ssi, 3 * D, 4 * D)
            self._gemm(f, ln[p + "ff.ff.0.proj"], ws.u[:V], x_scale=fsc, kind=_lib.EPI_SWIGLU,
                       amax_out=ws.amax[s0 + 5:s0 + 6] if self.fp8 else None)
            ua, usc = self._quant(ws, ws.u[:V], None if ws.u8 is None else ws.u8[:V], s0 + 5)
            self._gemm(ua, ln[p + "ff.ff.2"], hv, x_scale=usc, kind=_lib.EPI_GATED_RESIDUAL, residual=hv,
                       gate=ssi[:, 5 * D:6 * D], row_batch=rb[:V])

        # ---- drop memory tokens, project_out (postprocess conv folded) (transformer.py:1265-1267, dit.py:297-304)
        ops.convert(h, ws.hb, src_rows=ws.lat_rows)
        self._gemm(ws.hb, ln["project_out"], ws.out)


class GraphedStep:
    """One denoiser forward captured in a CUDA graph, replayed with new inputs copied into static buffers.

    Mirrors the reference TensorRT runner's graph-captured DiT step (optimized/tensorRT/scripts/
    sa3_trt_core.py:511-694): all kernel launches of the step replay with no host work.
    """

    def __init__(self, engine: DiTEngine, inputs, cfg_scale: float, apg_scale: float, padding_mask=None):
        self.engine = engine
        self.static = [None if a is None else a.to(engine.dev).clone() for a in inputs]
        self.cfg_scale, self.apg_scale = cfg_scale, apg_scale
        self.padding_mask = None if padding_mask is None else padding_mask.to(engine.dev).clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                engine.forward(*self.static, cfg_scale=cfg_scale, apg_scale=apg_scale, padding_mask=self.padding_mask)
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = engine.forward(*self.static, cfg_scale=cfg_scale, apg_scale=apg_scale,
                                      padding_mask=self.padding_mask)
        # the graph replays into these buffers: keep them alive even after the engine switches to another shape
        self.workspace, self.rope = engine.ws, engine.rope

    def __call__(self, x, t, cross_attn_cond=None, global_embed=None, local_add_cond=None) -> torch.Tensor:
        for dst, src in zip(self.static, (x, t, cross_attn_cond, global_embed, local_add_cond)):
            if dst is not None:
                dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.out
