"""Host-side logic of PagedDecodeGraph that needs no GPU."""

import pytest

from mini_llm_runtime_b200.decode_graph import PagedDecodeGraph


@pytest.mark.parametrize("layers", [1, 2, 3, 4, 5, 9, 24, 28, 64])
def test_copy_chunks_cover_the_layers_in_order(layers):
    chunks = PagedDecodeGraph.copy_chunks(layers)
    assert chunks[0][0] == 0 and chunks[-1][1] == layers
    assert all(b > a for a, b in chunks)
    assert all(chunks[i][1] == chunks[i + 1][0] for i in range(len(chunks) - 1))
    assert max(b - a for a, b in chunks) <= max(PagedDecodeGraph.COPY_CHUNK_LAYERS,
                                                 PagedDecodeGraph.EDGE_CHUNK_LAYERS)


def test_copy_chunks_edges_are_short():
    # The first chunk's inputs and the last chunk's outputs are not hidden
    # under any kernel, so they carry the fewest layers.
    chunks = PagedDecodeGraph.copy_chunks(24)
    edge = PagedDecodeGraph.EDGE_CHUNK_LAYERS
    assert chunks[0] == (0, edge) and chunks[-1] == (24 - edge, 24)
