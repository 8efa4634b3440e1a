"""Time-chunked decode of long utterances (exact, no communication).

The decoder is causal with a finite left receptive field: an output sample
depends only on latent frames at or before its own frame, back to a fixed
distance set by the architecture.  A chunk of frames [c0, c1) decoded from
the latent window [c0 - H, c1) (H >= the receptive field, in frames)
reproduces the full decode's samples [c0 * hop, c1 * hop): the H halo frames
supply all the history, and the window's own start (zero padding) only
affects the halo's samples, which are dropped.  At the utterance start
(c0 = 0) the window starts at frame 0 with the true zero padding.

So a long utterance splits over GPUs (or over several decodes on one GPU,
bounding activation memory) with no exchange: every part reads its latent
window and writes its own sample range.

Receptive field (reference src/audio-vae.cpp: the causal depthwise convs of
``decode_tensor_l2`` and ``residual_unit_forward_l2`` pad 6*d on the left,
the transposed convs reach one input frame back, ``final_conv_k7_l2_custom``
reads 6 samples back):
  model.0 k7                 6 latent frames
  block b (stride s_b, rate R_b = s_1 * ... * s_b samples per frame):
    transposed conv          1 input sample  = 1 / R_{b-1} frames
    residual units d=1,3,9   6 * (1+3+9) = 78 samples at R_b
  final conv k7              6 samples at R_last
For rates (8, 8, 5, 2): 18.49 frames, so H = 19 is the least exact halo.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

DILATIONS = (1, 3, 9)
KERNEL = 7


def receptive_field_frames(rates=(8, 8, 5, 2), kernel: int = KERNEL, dilations=DILATIONS) -> float:
    """Left receptive field of one output sample, in latent frames."""
    reach = kernel - 1  # model.0 depthwise conv at the latent rate
    rf = float(reach)
    r = 1
    for s in rates:
        rf += 1.0 / r  # transposed conv: the previous input sample
        r *= s
        rf += (kernel - 1) * sum(dilations) / r  # three dilated residual units
    rf += (kernel - 1) / r  # final conv
    return rf


def min_halo(rates=(8, 8, 5, 2)) -> int:
    """Smallest whole number of halo frames that makes a chunk exact."""
    return math.ceil(receptive_field_frames(rates))


def encoder_receptive_field_frames(rates=(2, 5, 8, 8), kernel: int = KERNEL, dilations=DILATIONS) -> float:
    """Left reach of one latent frame of the encoder (in latent frames): the
    encoder is causal as well (reference encode_tensor / encoder_block_forward,
    src/audio-vae.cpp:553-570, 640-650: every conv pads on the left only),
    so a waveform window that starts this far before the frames it keeps
    reproduces them.  In samples: the head conv reads 6 back; block b at r_b
    samples per position (r_1 = 1) adds its three dilated residual units
    (6 * (1+3+9) positions) and its strided conv's left pad (2 * ceil(s/2)
    positions); fc_mu reads 2 frames back."""
    reach = kernel - 1
    r = 1
    for s in rates:
        reach += r * ((kernel - 1) * sum(dilations) + 2 * ((s + 1) // 2))
        r *= s
    reach += 2 * r
    return reach / r


def min_encoder_halo(rates=(2, 5, 8, 8)) -> int:
    """Smallest whole number of halo frames that makes an encoder chunk exact."""
    return math.ceil(encoder_receptive_field_frames(rates))


@dataclass(frozen=True)
class Chunk:
    start: int  # first latent frame decoded (window start, includes the halo)
    keep: int   # first frame whose samples are kept (>= start)
    end: int    # one past the last frame

    @property
    def frames(self) -> int:
        return self.end - self.start

    @property
    def halo(self) -> int:
        return self.keep - self.start


def split(T: int, parts: int, halo: int) -> list[Chunk]:
    """Splits frames [0, T) into `parts` contiguous kept ranges of near-equal
    length (the first ones one frame longer), each with up to `halo` frames
    of left context.  Empty parts are omitted (parts > T)."""
    if T <= 0 or parts <= 0 or halo < 0:
        raise ValueError("split needs T > 0, parts > 0, halo >= 0")
    base, extra = divmod(T, parts)
    out, c0 = [], 0
    for p in range(parts):
        n = base + (1 if p < extra else 0)
        if n == 0:
            continue
        out.append(Chunk(max(0, c0 - halo), c0, c0 + n))
        c0 += n
    return out


def chunks_of(T: int, chunk: int, halo: int) -> list[Chunk]:
    """Kept ranges of `chunk` frames (the last one shorter), each with up to
    `halo` frames of left context."""
    if T <= 0 or chunk <= 0 or halo < 0:
        raise ValueError("chunks_of needs T > 0, chunk > 0, halo >= 0")
    return [Chunk(max(0, c0 - halo), c0, min(T, c0 + chunk)) for c0 in range(0, T, chunk)]
