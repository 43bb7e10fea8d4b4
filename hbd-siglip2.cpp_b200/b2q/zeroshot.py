"""Zero-shot image-text scoring sharded over ranks.

The reference scores one request at a time on one GPU: encode the image(s),
encode the prompts, L2-normalise both and apply the sigmoid head
(src/siglip2_score.cpp:78-134, driven by the classify route at
src/siglip2_server.cpp:763-880).  Here a whole image set is scored against a
prompt set with both sets split over the ranks: every rank encodes its
contiguous share of the images and of the prompts, the prompt embeddings are
all-gathered so that every rank holds all of them, each rank scores its own
images against every prompt, and the score rows are gathered in image order.
Images and prompts are independent, so the only exchanges are those two
gathers (NCCL on the GPU box, gloo in the CPU tests).

The encoders and the scorer are passed in, so that the same orchestration
runs the CUDA towers in bench.py and stand-ins in the CPU tests.
"""
from __future__ import annotations

from typing import Callable

from .shard import gather_in_order, shard_rows


def zero_shot(encode_images: Callable, encode_texts: Callable, score: Callable, n_images: int, n_prompts: int,
              rank: int = 0, world: int = 1, group=None, timings: dict | None = None):
    """Scores of all n_images images against all n_prompts prompts.

    encode_images(rows: range) -> [len(rows), H] embeddings of those images;
    encode_texts(rows: range)  -> [len(rows), H] embeddings of those prompts;
    score(img, txt)            -> [len(img), len(txt)] scores (a torch tensor).
    Returns the [n_images, n_prompts] score matrix, in image order, on every
    rank.  With world == 1 no collective is issued.  `timings`, when given,
    receives CUDA-event pairs ("encode", "gather_text", "score",
    "gather_scores") recorded on the current stream when CUDA is in use."""
    import torch

    img_rows = shard_rows(n_images, rank, world)
    txt_rows = shard_rows(n_prompts, rank, world)
    use_events = timings is not None and torch.cuda.is_available()

    def mark(name):
        if use_events:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            timings.setdefault(name, []).append(ev)

    mark("start")
    img = encode_images(img_rows)
    txt_local = encode_texts(txt_rows)
    mark("encoded")
    if world > 1:
        txt = gather_in_order(txt_local, list(txt_rows), n_prompts, group=group)
    else:
        txt = txt_local
    mark("text_gathered")
    local = score(img, txt)
    mark("scored")
    if world > 1:
        out = gather_in_order(local, list(img_rows), n_images, group=group)
    else:
        out = local
    mark("done")
    return out
