"""GPU-resident greedy decode-step primitives around the Q8 projections
(graph_helpers.metal:12-178, :354-388, :785-821): with the token history, the
position counters and the logits in device memory, a whole token step runs with
no host round trip and replays as a CUDA graph.

Thin wrappers of the C ABI (madi_emb_lookup_q8, madi_emb_pos_q8, madi_argmax_conf,
madi_logit_filter, madi_logit_filter_rows, madi_suppress_rows, madi_step_advance,
madi_decode_tail, madi_shard_decode_tail, madi_merge_shard_tail) on torch CUDA tensors.
"""
import ctypes
from typing import Optional

import torch

from . import _lib
from .q8 import Q8Weight, _stream


def emb_lookup_q8(emb: Q8Weight, tokens: torch.Tensor, pos: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Token embeddings from a Q8 table: tokens u32 [m][len] with positions pos u32 [m]
    (row s uses tokens[s][pos[s]]), or tokens u32 [m] directly when pos is None.
    Returns f32 [m][dim]."""
    if tokens.dtype != torch.int32 and tokens.dtype != torch.uint32:
        raise TypeError("tokens must be 32-bit")
    if pos is None:
        m, tok_stride, tok_len = tokens.numel(), 1, 1
    else:
        if tokens.dim() != 2 or not tokens.is_contiguous():
            raise ValueError("tokens must be a contiguous [m][len] tensor when pos is given")
        m, tok_len = tokens.shape
        tok_stride = tok_len
        if pos.numel() != m:
            raise ValueError("pos must have one entry per slot")
    if out is None:
        out = torch.empty((m, emb.k), dtype=torch.float32, device=tokens.device)
    h = emb.handle()
    rc = _lib.load().madi_emb_lookup_q8(ctypes.byref(h), tokens.data_ptr(), None if pos is None else pos.data_ptr(), m,
                                        tok_stride, tok_len, out.data_ptr(), _stream(stream))
    _lib.check(rc, "madi_emb_lookup_q8")
    return out


def emb_pos_q8(emb: Q8Weight, tokens: torch.Tensor, pos: torch.Tensor, pos_emb: torch.Tensor,
               out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """emb_lookup_q8 plus the positional embedding in one launch: tokens u32 [m][len],
    pos u32 [m] on the device, pos_emb f32 [max_pos][dim]; row s is
    emb(tokens[s][pos[s]]) + pos_emb[pos[s]].  Returns f32 [m][dim]."""
    if tokens.dtype not in (torch.int32, torch.uint32) or tokens.dim() != 2 or not tokens.is_contiguous():
        raise ValueError("tokens must be a contiguous 32-bit [m][len] tensor")
    m, tok_len = tokens.shape
    if pos.numel() != m:
        raise ValueError("pos must have one entry per slot")
    if pos_emb.dtype != torch.float32 or pos_emb.dim() != 2 or pos_emb.shape[1] != emb.k or not pos_emb.is_contiguous():
        raise ValueError("pos_emb must be a contiguous f32 [max_pos][dim] tensor")
    if out is None:
        out = torch.empty((m, emb.k), dtype=torch.float32, device=tokens.device)
    h = emb.handle()
    rc = _lib.load().madi_emb_pos_q8(ctypes.byref(h), tokens.data_ptr(), pos.data_ptr(), m, tok_len, tok_len,
                                     pos_emb.data_ptr(), pos_emb.shape[0], out.data_ptr(), _stream(stream))
    _lib.check(rc, "madi_emb_pos_q8")
    return out


def argmax_conf(logits: torch.Tensor, tokens: torch.Tensor, pos: torch.Tensor, conf: Optional[torch.Tensor] = None,
                stream=None) -> None:
    """tokens[s][pos[s]] = argmax(logits[s]) (and conf[s][pos[s]] = its softmax
    probability) for every slot with pos[s] < tokens.shape[1]."""
    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous f32 [m][vocab] tensor")
    m, vocab = logits.shape
    if tokens.dim() != 2 or tokens.shape[0] != m or not tokens.is_contiguous():
        raise ValueError("tokens must be a contiguous [m][max_len] tensor")
    max_len = tokens.shape[1]
    if conf is not None and (conf.shape != tokens.shape or conf.dtype != torch.float32 or not conf.is_contiguous()):
        raise ValueError("conf must be f32 shaped like tokens")
    rc = _lib.load().madi_argmax_conf(logits.data_ptr(), m, vocab, tokens.data_ptr(),
                                      None if conf is None else conf.data_ptr(), pos.data_ptr(), max_len, max_len,
                                      _stream(stream))
    _lib.check(rc, "madi_argmax_conf")


def logit_filter(logits: torch.Tensor, past: torch.Tensor, step: torch.Tensor, sample_begin: int,
                 no_repeat_ngram: int = 0, stream=None) -> None:
    """logit_filter_indirect on one f32 logits row, in place; step is a device u32 [1]."""
    rc = _lib.load().madi_logit_filter(logits.data_ptr(), logits.numel(), past.data_ptr(), past.numel(),
                                       step.data_ptr(), int(sample_begin), int(no_repeat_ngram), _stream(stream))
    _lib.check(rc, "madi_logit_filter")


def logit_filter_rows(logits: torch.Tensor, past: torch.Tensor, pos: torch.Tensor, sample_begin: int,
                      no_repeat_ngram: int = 0, stream=None) -> None:
    """logit_filter on every row of logits f32 [m][vocab] in one launch: row s uses
    the history past[s] (u32 [m][len]) and the step pos[s] (device u32 [m])."""
    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous f32 [m][vocab] tensor")
    m, vocab = logits.shape
    if past.dim() != 2 or past.shape[0] != m or not past.is_contiguous() or pos.numel() != m:
        raise ValueError("past must be a contiguous [m][len] tensor and pos hold one step per row")
    rc = _lib.load().madi_logit_filter_rows(logits.data_ptr(), m, vocab, past.data_ptr(), past.shape[1], past.shape[1],
                                            pos.data_ptr(), int(sample_begin), int(no_repeat_ngram), _stream(stream))
    _lib.check(rc, "madi_logit_filter_rows")


def suppress_rows(logits: torch.Tensor, ids: torch.Tensor, stream=None) -> None:
    """suppress_list on every row of logits f32 [m][vocab]: the token ids (device
    u32 [n]) get -3.4e38."""
    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous f32 [m][vocab] tensor")
    if ids.dtype not in (torch.int32, torch.uint32) or not ids.is_contiguous():
        raise ValueError("ids must be a contiguous 32-bit tensor")
    m, vocab = logits.shape
    _lib.check(_lib.load().madi_suppress_rows(logits.data_ptr(), m, vocab, ids.data_ptr(), ids.numel(),
                                              _stream(stream)), "madi_suppress_rows")


def decode_tail(logits: torch.Tensor, tokens: torch.Tensor, pos: torch.Tensor, conf: Optional[torch.Tensor] = None,
                sample_begin: int = 1, no_repeat_ngram: int = 0, suppress: Optional[torch.Tensor] = None,
                stream=None) -> None:
    """step_advance, logit_filter_rows, suppress_rows and argmax_conf in one launch:
    pos[s] += 1, logits [m][vocab] filtered in place, tokens[s][pos[s]] (and conf) written."""
    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous f32 [m][vocab] tensor")
    m, vocab = logits.shape
    if tokens.dim() != 2 or tokens.shape[0] != m or not tokens.is_contiguous() or pos.numel() != m:
        raise ValueError("tokens must be a contiguous [m][max_len] tensor and pos hold one position per slot")
    max_len = tokens.shape[1]
    if conf is not None and (conf.shape != tokens.shape or conf.dtype != torch.float32 or not conf.is_contiguous()):
        raise ValueError("conf must be f32 shaped like tokens")
    nsup = 0 if suppress is None else suppress.numel()
    rc = _lib.load().madi_decode_tail(logits.data_ptr(), m, vocab, tokens.data_ptr(), max_len, max_len,
                                      pos.data_ptr(), None if conf is None else conf.data_ptr(), int(sample_begin),
                                      int(no_repeat_ngram), None if suppress is None else suppress.data_ptr(), nsup,
                                      _stream(stream))
    _lib.check(rc, "madi_decode_tail")


def step_advance(pos: torch.Tensor, stream=None) -> None:
    """pos[s] += 1 on the device."""
    _lib.check(_lib.load().madi_step_advance(pos.data_ptr(), pos.numel(), _stream(stream)), "madi_step_advance")


def shard_decode_tail(logits: torch.Tensor, h0: int, vocab: int, tokens: torch.Tensor, pos: torch.Tensor,
                      part: torch.Tensor, sample_begin: int = 1, no_repeat_ngram: int = 0,
                      suppress: Optional[torch.Tensor] = None, stream=None) -> None:
    """decode_tail over one column shard of the vocab head: logits [m][n] hold the
    global token ids [h0, h0 + n) for all m rows of the job; tokens [m][max_len] and
    pos [m] are the rows' shared history (read only).  Writes part [m][4] f32 =
    (max, global index as u32 bits, exp sum against the max, 0) per row."""
    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous f32 [m][n] tensor")
    m, n = logits.shape
    if tokens.dim() != 2 or tokens.shape[0] != m or not tokens.is_contiguous() or pos.numel() != m:
        raise ValueError("tokens must be a contiguous [m][max_len] tensor and pos hold one position per row")
    if part.dtype != torch.float32 or tuple(part.shape) != (m, 4) or not part.is_contiguous():
        raise ValueError("part must be a contiguous f32 [m][4] tensor")
    max_len = tokens.shape[1]
    nsup = 0 if suppress is None else suppress.numel()
    rc = _lib.load().madi_shard_decode_tail(logits.data_ptr(), m, n, int(h0), int(vocab), tokens.data_ptr(), max_len,
                                            max_len, pos.data_ptr(), int(sample_begin), int(no_repeat_ngram),
                                            None if suppress is None else suppress.data_ptr(), nsup, part.data_ptr(),
                                            _stream(stream))
    _lib.check(rc, "madi_shard_decode_tail")


def merge_shard_tail(parts: torch.Tensor, tokens: torch.Tensor, pos: torch.Tensor,
                     conf: Optional[torch.Tensor] = None, stream=None) -> None:
    """The rest of decode_tail from the all-gathered shard parts [world][m][4]:
    pos[row] += 1, tokens[row][pos[row]] and conf[row][pos[row]] written."""
    if parts.dim() != 3 or parts.shape[2] != 4 or parts.dtype != torch.float32 or not parts.is_contiguous():
        raise ValueError("parts must be a contiguous f32 [world][m][4] tensor")
    world, m, _ = parts.shape
    if tokens.dim() != 2 or tokens.shape[0] != m or not tokens.is_contiguous() or pos.numel() != m:
        raise ValueError("tokens must be a contiguous [m][max_len] tensor and pos hold one position per row")
    if conf is not None and (conf.shape != tokens.shape or conf.dtype != torch.float32 or not conf.is_contiguous()):
        raise ValueError("conf must be f32 shaped like tokens")
    max_len = tokens.shape[1]
    rc = _lib.load().madi_merge_shard_tail(parts.data_ptr(), world, m, tokens.data_ptr(), max_len, max_len,
                                           pos.data_ptr(), None if conf is None else conf.data_ptr(), _stream(stream))
    _lib.check(rc, "madi_merge_shard_tail")
