"""Embeddings (reference: tinytron/model/modules/emb.py:4-6)."""
import torch.nn as nn

TextEmbedding = nn.Embedding


class ImgEmbedding(nn.Module):
    """Placeholder kept for API parity: the reference exports ``ImgEmbedding = ...``
    without an implementation."""

    def __init__(self, *args, **kwargs):
        raise NotImplementedError("ImgEmbedding is a placeholder in Tinytron and has no implementation")
