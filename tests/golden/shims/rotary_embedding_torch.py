"""Test-only, NON-functional stand-in for ``rotary-embedding-torch``.

The rotary arithmetic lives in that third-party package, whose source is not
available here, so rotary numerics are unpinned. Importing works (the
reference imports these names at module load); constructing or applying a
rotary embedding raises, so no fixture can silently depend on it.
"""


class RotaryEmbedding:
    def __init__(self, *args, **kwargs):
        raise NotImplementedError("rotary-embedding-torch is not installed; rotary parity is unpinned")


def apply_rotary_emb(*args, **kwargs):
    raise NotImplementedError("rotary-embedding-torch is not installed; rotary parity is unpinned")
