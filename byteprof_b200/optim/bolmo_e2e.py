"""End-to-end greedy byte decoding of a random-init Bolmo-1B-shaped model on the sm_100a kernels.

Bolmo's remote model code and weights are not part of byteprof, so the model is defined here, with
the shapes of the end-to-end benchmark configuration and weights ~ N(0, 0.02) (norm weights 1 + N(0, 0.02)):
  * local encoder: byte embedding 512 x 2048 -> one mLSTM layer (bolmo_local.LocalLayer: 4 heads x 512,
    forget bias +3, gate soft cap 15, SwiGLU 2816) -> RMSNorm -> e;
  * boundary predictor: sigmoid(w_b . e) >= 0.5 (a 2048 -> 1 linear); patch vector P = W_p e;
  * global model, once per patch on P at patch position t: 16 OLMo-2 blocks (d 2048, 16 heads x 128; q and
    k RMSNorm over d; rotary embedding, theta 500000; attention over a static KV cache; the attention and
    MLP outputs RMS-normalised before each residual add; SwiGLU 8192), then the decoder's initial RMSNorm
    gives the patch value (byteprof/optim/bolmo_loop.py:58-61 does the same with dec.initial_norm);
  * local decoder: W_in e + patch value -> one mLSTM layer -> RMSNorm -> LM head 2048 -> 512 -> argmax.
The loop is byteprof's minimal loop (byteprof/optim/bolmo_loop.py:1-20, 182-207; bolmo.py:47-136): per
byte the encoder, the global step only when the previous step flagged a boundary (the first byte opens a
patch), the decoder, then one device-to-host read of (token, boundary flag): the only synchronisation.
Each byte is one CUDA graph launch (encoder + decoder, or encoder + global step + decoder). Every projection is a skinny GEMM of this library (M = 1), the mLSTM steps are
the fused scan, and the glue between them is the fused kernels of `decode_ops`. By default the global
step is one persistent kernel (decode_ops.GlobStep, csrc/glob_step.cu); fused_glob=False runs it kernel
by kernel (GlobalBlock.step). fused_local chooses which local steps run as one persistent kernel
(decode_ops.LocStep, csrc/loc_step.cu): True (the default: both; on B200 the encoder step takes 46 us
against 57 kernel by kernel, the decoder step 54 against 61), "enc", "dec" or False (neither).

precision="fp32" is the exactness mode: the same weights (bf16) with fp32 activations, fp32 KV caches
and no rounding of any intermediate to bf16, kernel by kernel (skinny GEMMs read x as fp32, the glue
kernels and the scan run their fp32 forms). It decodes the bytes that exact arithmetic on the same
weights decodes, so it pins the whole model end to end; the default "bf16" mode is the fast one.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from .. import _lib

from .bolmo_local import LocalLayer, rmsnorm
from .decode_ops import (DecodeAttention, GlobStep, LocStep, add_norm, decode_finish, embed_rmsnorm, norm_add,
                         rope_tables, swiglu)
from .skinny import skinny_mm

EPS = 1e-6


def _rnd(gen, device, *shape, std=0.02):
    return (torch.randn(*shape, generator=gen, device=device) * std).to(torch.bfloat16)


def _norm_w(gen, device, *shape):
    return (1.0 + torch.randn(*shape, generator=gen, device=device) * 0.02).to(torch.bfloat16)


class GlobalBlock:
    """One OLMo-2 block for single-position decoding with a static KV cache."""

    def __init__(self, d: int, nh: int, ffn: int, max_pos: int, gen: torch.Generator, device: torch.device,
                 act_dtype: torch.dtype = torch.bfloat16):
        self.d, self.nh, self.ffn = d, nh, ffn
        self.w_qkv = _rnd(gen, device, 3 * d, d)
        self.q_norm = _norm_w(gen, device, d)
        self.k_norm = _norm_w(gen, device, d)
        self.w_o = _rnd(gen, device, d, d)
        self.attn_norm = _norm_w(gen, device, d)
        self.w_gu = _rnd(gen, device, 2 * ffn, d)
        self.w_down = _rnd(gen, device, d, ffn)
        self.mlp_norm = _norm_w(gen, device, d)
        self.attn = DecodeAttention(nh, d // nh, max_pos, device, dtype=act_dtype)

    def step(self, x: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """x [1, d] (the activation dtype) at patch position `pos` (device int64) -> the block's output [1, d]."""
        att = self.attn(skinny_mm(x, self.w_qkv), self.q_norm, self.k_norm, cos, sin, pos, EPS)
        h = add_norm(skinny_mm(att, self.w_o), x, self.attn_norm, EPS)
        dn = skinny_mm(swiglu(skinny_mm(h, self.w_gu)), self.w_down)
        return add_norm(dn, h, self.mlp_norm, EPS)


class BolmoDecoder:
    """The byte model with its per-byte CUDA graphs and the greedy decode loop (batch 1)."""

    def __init__(self, device: torch.device | str = "cuda", seed: int = 0, d: int = 2048, vocab: int = 512,
                 local_heads: int = 4, local_dh: int = 512, local_ffn: int = 2816, global_layers: int = 16,
                 global_heads: int = 16, global_ffn: int = 8192, max_patches: int = 1024,
                 rope_theta: float = 500000.0, fused_glob: bool = True, fused_local: bool | str = True,
                 precision: str = "bf16"):
        if precision not in ("bf16", "fp32"):
            raise ValueError(f"precision must be 'bf16' or 'fp32', got {precision!r}")
        if fused_local not in (False, True, "enc", "dec"):
            raise ValueError(f"fused_local must be False, True, 'enc' or 'dec', got {fused_local!r}")
        act = torch.bfloat16 if precision == "bf16" else torch.float32
        if act == torch.float32:  # the persistent kernels run bf16 activations only
            fused_glob = fused_local = False
        self.precision, self.act = precision, act
        device = torch.device(device)
        gen = torch.Generator(device=device).manual_seed(seed)
        self.device, self.d, self.vocab, self.max_patches = device, d, vocab, max_patches
        self.embed = _rnd(gen, device, vocab, d)
        self.enc = LocalLayer(d, local_heads, local_dh, local_ffn, gen, device, smax=1, act_dtype=act)
        self.enc_norm = _norm_w(gen, device, d)
        self.w_boundary = _rnd(gen, device, 1, d)
        self.w_patch = _rnd(gen, device, d, d)
        self.blocks = [GlobalBlock(d, global_heads, global_ffn, max_patches, gen, device, act_dtype=act)
                       for _ in range(global_layers)]
        self.dec_in_norm = _norm_w(gen, device, d)
        self.w_in = _rnd(gen, device, d, d)
        self.dec = LocalLayer(d, local_heads, local_dh, local_ffn, gen, device, smax=1, act_dtype=act)
        self.final_norm = _norm_w(gen, device, d)
        self.lm_head = _rnd(gen, device, vocab, d)
        self.cos, self.sin = rope_tables(max_patches, d // global_heads, rope_theta, device)
        # per-byte device buffers (graph inputs and outputs)
        self.byte = torch.zeros(1, dtype=torch.long, device=device)
        self.pos = torch.zeros(1, dtype=torch.long, device=device)  # the next patch position
        self.e = torch.zeros(1, d, dtype=act, device=device)
        self.patch = torch.zeros(1, d, dtype=act, device=device)
        self.value = torch.zeros(1, d, dtype=act, device=device)
        self.boundary_logit = torch.zeros(1, 1, dtype=torch.float32, device=device)
        self.logits = torch.zeros(1, vocab, dtype=torch.float32, device=device)
        self.out = torch.zeros(2, dtype=torch.long, device=device)  # [token, boundary flag]
        self.graphs: dict[str, torch.cuda.CUDAGraph] = {}
        self.parity = 0  # which n / m buffers of the local layers hold the current state
        self.patches = 0  # patch positions used (host count)
        self._pin_byte = torch.zeros(1, dtype=torch.long).pin_memory()
        self._pin_out = torch.zeros(2, dtype=torch.long).pin_memory()
        self._byte_np, self._out_np = self._pin_byte.numpy(), self._pin_out.numpy()  # host views, no torch ops
        # the global step as one persistent kernel, or kernel by kernel (GlobalBlock.step)
        self.fused_glob = fused_glob
        self.glob_kernel = GlobStep(self.blocks, self.dec_in_norm, self.cos, self.sin, max_patches, EPS) \
            if fused_glob else None
        # the local steps as one persistent kernel each, or kernel by kernel (LocalLayer.step)
        self.enc_kernel = LocStep(self.enc) if fused_local in (True, "enc") else None
        self.dec_kernel = LocStep(self.dec) if fused_local in (True, "dec") else None

    def weights(self) -> dict[str, torch.Tensor]:
        """Every parameter by name (the CPU oracle rebuilds the model from these)."""
        w = {"embed": self.embed, "enc_norm": self.enc_norm, "w_boundary": self.w_boundary, "w_patch": self.w_patch,
             "dec_in_norm": self.dec_in_norm, "w_in": self.w_in, "final_norm": self.final_norm,
             "lm_head": self.lm_head}
        for name, layer in (("enc", self.enc), ("dec", self.dec)):
            for a in ("norm1", "w_qkvo", "w_if", "b_if", "mh_norm", "w_out", "norm2", "w_gu", "w_down"):
                w[f"{name}.{a}"] = getattr(layer, a)
        for i, b in enumerate(self.blocks):
            for a in ("w_qkv", "q_norm", "k_norm", "w_o", "attn_norm", "w_gu", "w_down", "mlp_norm"):
                w[f"glob{i}.{a}"] = getattr(b, a)
        return w

    # ---- the three per-byte pieces (device only, graph-capturable) ----
    def enc_step(self, parity: int) -> None:
        if self.enc_kernel is not None:
            self.enc_kernel.enc(parity, self.embed, self.byte, self.enc_norm, self.w_patch, self.w_boundary, self.e,
                                self.patch, self.boundary_logit)
            return
        if self.act == torch.bfloat16:
            h, x = embed_rmsnorm(self.embed, self.byte, self.enc.norm1, EPS)
        else:
            h = self.embed.index_select(0, self.byte).to(self.act)
            x = rmsnorm(h, self.enc.norm1, EPS)
        self.enc.step(h, x, parity, out_norm=self.enc_norm, want_sum=False, out=self.e)
        skinny_mm(self.e, self.w_patch, out=self.patch)
        skinny_mm(self.e, self.w_boundary, out=self.boundary_logit)

    def encdec_step(self, parity: int) -> None:
        """enc_step and dec_step of a byte that opens no patch as one launch (the persistent local steps only);
        the same results as the two, bit for bit."""
        self.enc_kernel.encdec(self.dec_kernel, parity, self.embed, self.byte, self.enc_norm, self.w_patch,
                               self.w_boundary, self.e, self.patch, self.boundary_logit, self.value, self.w_in,
                               self.final_norm, self.lm_head, self.logits, self.out)

    def glob_step(self) -> None:
        if self.glob_kernel is not None:
            self.glob_kernel(self.patch, self.value, self.pos)  # writes value, advances pos
            return
        x = self.patch
        for blk in self.blocks:
            x = blk.step(x, self.pos, self.cos, self.sin)
        rmsnorm(x, self.dec_in_norm, EPS, out=self.value)
        self.pos.add_(1)

    def dec_step(self, parity: int) -> None:
        if self.dec_kernel is not None:
            self.dec_kernel.dec(parity, self.e, self.value, self.w_in, self.final_norm, self.lm_head,
                                self.boundary_logit, self.logits, self.out)
            return
        h, x = norm_add(skinny_mm(self.e, self.w_in), self.value, self.dec.norm1, EPS)
        _, xf = self.dec.step(h, x, parity, out_norm=self.final_norm, want_sum=False)
        skinny_mm(xf, self.lm_head, out=self.logits)
        decode_finish(self.logits, self.boundary_logit, self.out)

    # ---- state ----
    def reset(self) -> None:
        self.enc.reset()
        self.dec.reset()
        self.pos.zero_()
        self.value.zero_()
        for blk in self.blocks:
            blk.attn.reset()
        self.parity = 0
        self.patches = 0

    def _pieces(self):
        return (("enc0", lambda: self.enc_step(0)), ("enc1", lambda: self.enc_step(1)), ("glob", self.glob_step),
                ("dec0", lambda: self.dec_step(0)), ("dec1", lambda: self.dec_step(1)))

    def _bytes(self):
        """The whole work of one byte as one piece, per state parity: the byte's copy in from pinned memory,
        encoder and decoder, or encoder, global step and decoder when the byte opens a patch, and the copy
        of (token, boundary flag) out to pinned memory (one graph launch per byte, no gaps between graphs)."""
        def one(p: int, patch: bool):
            def fn():
                self.byte.copy_(self._pin_byte, non_blocking=True)
                if not patch and self.enc_kernel is not None and self.dec_kernel is not None:
                    self.encdec_step(p)  # no global step between them: one launch for both
                    self._pin_out.copy_(self.out, non_blocking=True)
                    return
                self.enc_step(p)
                if patch:
                    self.glob_step()
                self.dec_step(p)
                self._pin_out.copy_(self.out, non_blocking=True)
            return fn
        return tuple((f"{'patch' if patch else 'byte'}{p}", one(p, patch)) for p in (0, 1) for patch in (False, True))

    def capture(self) -> None:
        """One CUDA graph per piece and state parity (the pieces alone, for timing them, and each byte's whole
        work, which `launch` replays). The warm-up runs go through the same buffers and are undone by `reset`
        (capture before decoding)."""
        s_ = torch.cuda.Stream()
        s_.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_):
            for _, fn in self._pieces():
                fn()
        torch.cuda.current_stream().wait_stream(s_)
        for name, fn in self._pieces() + self._bytes():
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            self.graphs[name] = g
        torch.cuda.synchronize()
        self.reset()

    def launch(self, b: int, new_patch: bool) -> None:
        """Queue one byte (encoder, the global model if a patch starts here, decoder); no sync. The byte goes
        through one pinned host word that the queued work reads when it runs, so synchronise (as `feed` does)
        before the next launch."""
        if not 0 <= b < self.vocab:
            raise ValueError(f"byte id {b} outside the vocabulary")
        if new_patch and self.patches >= self.max_patches:
            raise RuntimeError(f"more than {self.max_patches} patches: the static KV cache is full")
        p = self.parity
        self._byte_np[0] = b
        whole = self.graphs.get(f"{'patch' if new_patch else 'byte'}{p}")
        if whole is not None:
            whole.replay()  # copies the byte in and (token, flag) out itself
        else:
            self.byte.copy_(self._pin_byte, non_blocking=True)
            self.enc_step(p)
            if new_patch:
                self.glob_step()
            self.dec_step(p)
            self._pin_out.copy_(self.out, non_blocking=True)
        if new_patch:
            self.patches += 1
        self.parity = 1 - p

    def feed(self, b: int, new_patch: bool) -> tuple[int, bool]:
        """One byte, then the step's single synchronisation; returns (greedy token, boundary flag)."""
        self.launch(b, new_patch)
        torch.cuda.current_stream().synchronize()
        return int(self._out_np[0]), bool(self._out_np[1])

    def steps(self, n: int, bytes_=None, patches=None, first_byte: int = 0, first_patch: bool = True):
        """n bytes through the captured per-byte graphs in the native loop (bp_decode_loop), one synchronisation
        per byte. Step i feeds bytes_[i] (or first_byte, then the previous step's greedy token) and opens a
        patch when patches[i] (or first_patch, then the previous step's boundary flag). Returns (tokens,
        boundary flags, patch starts fed, wall seconds of the loop)."""
        if not self.graphs:
            raise RuntimeError("steps() runs the captured graphs: call capture() first")
        if bytes_ is not None:
            bytes_ = np.ascontiguousarray(bytes_, dtype=np.int64)
            if bytes_.shape != (n,) or (n and (bytes_.min() < 0 or bytes_.max() >= self.vocab)):
                raise ValueError(f"bytes_ must hold n byte ids in [0, {self.vocab})")
        elif not 0 <= first_byte < self.vocab:
            raise ValueError(f"byte id {first_byte} outside the vocabulary")
        if patches is not None:
            patches = np.ascontiguousarray(patches, dtype=np.int32)
            if patches.shape != (n,):
                raise ValueError("patches must hold n flags")
            need = int(patches.astype(bool).sum())
        else:
            need = n  # at most one patch per byte
        if self.patches + need > self.max_patches:
            raise RuntimeError(f"up to {self.patches + need} patches: more than the static KV cache's {self.max_patches}")
        execs = [self.graphs[f"{kind}{p}"].raw_cuda_graph_exec() for p in (0, 1) for kind in ("byte", "patch")]
        tokens, flags, wall = native_steps(execs, self._pin_byte, self._pin_out, n, bytes_, patches, first_byte,
                                           first_patch, self.parity, self.device)
        opened = patches.astype(bool).tolist() if patches is not None else \
            ([bool(first_patch)] + [bool(f) for f in flags[:n - 1]])[:n]
        self.patches += sum(opened)
        self.parity ^= n & 1
        return tokens.tolist(), [bool(f) for f in flags], opened, wall

    @torch.no_grad()
    def generate(self, prompt: list[int], n_new: int) -> tuple[list[int], list[bool]]:
        """Greedy decoding from the current state: the prompt bytes in order, then each predicted byte.
        Returns the n_new generated bytes and, for every byte fed, whether it opened a patch. Runs the
        captured graphs in the native loop when present, else byte by byte."""
        if not self.graphs:
            new_patch, opened, tok = True, [], 0
            for b in prompt:
                opened.append(new_patch)
                tok, new_patch = self.feed(b, new_patch)
            out = []
            for i in range(n_new):
                out.append(tok)
                if i + 1 < n_new:
                    opened.append(new_patch)
                    tok, new_patch = self.feed(tok, new_patch)
            return out, opened
        toks, flags, opened, _ = self.steps(len(prompt), bytes_=prompt, first_patch=True)
        if n_new <= 0:
            return [], opened
        out = [toks[-1]]
        if n_new > 1:
            gen, _, op2, _ = self.steps(n_new - 1, first_byte=toks[-1], first_patch=flags[-1])
            out += gen
            opened += op2
        return out, opened


def native_steps(execs, pin_byte: torch.Tensor, pin_out: torch.Tensor, n: int, bytes_, patches, first_byte: int,
                 first_patch: bool, parity: int, device) -> tuple[np.ndarray, np.ndarray, float]:
    """bp_decode_loop over four graph execs (index 2 * parity + patch) whose first node copies the pinned
    byte word in and whose last copies (token, flag) to the pinned pair. Returns (tokens, flags, wall s)."""
    arr = (ctypes.c_void_p * 4)(*execs)
    tokens = np.zeros(max(n, 1), np.int64)
    flags = np.zeros(max(n, 1), np.int32)
    wall = ctypes.c_double(0.0)
    with torch.cuda.device(device):
        _lib.call("bp_decode_loop", arr, pin_byte.data_ptr(), pin_out.data_ptr(),
                  None if bytes_ is None else bytes_.ctypes.data, None if patches is None else patches.ctypes.data,
                  n, int(first_byte), int(bool(first_patch)), int(parity), tokens.ctypes.data, flags.ctypes.data,
                  torch.cuda.current_stream(device).cuda_stream, ctypes.byref(wall))
    return tokens[:n], flags[:n], wall.value
