"""Expert-page layout (host side of the pager): a page is one (layer, expert) with
its gate, up and down codes, scales and biases back to back, in the order and
sizes astro_moe_pager_create documents."""
import numpy as np

from astronomical_b200 import paging, synthetic


def test_page_bytes_of_the_config1_block():
    # 3 * 2048 * 512 / 2 bytes of codes + 3 * 2048 * 512 / 64 * 2 * 2 of scales/biases
    assert paging.page_bytes(synthetic.CONFIGS[1]) == 1769472


def test_pack_expert_pages_layout():
    cfg = dict(synthetic.CONFIGS[0], experts=4, intermediate=128)
    layers = [synthetic.make_block_weights(cfg, seed=s) for s in (1, 2)]
    store = paging.pack_expert_pages(layers, pin=False).numpy()
    P = paging.page_bytes(cfg)
    assert store.shape == (2, 4, P)
    for li, w in enumerate(layers):
        for e in range(4):
            parts = [np.ascontiguousarray(w[k][e]).view(np.uint8).ravel() for k in
                     ("gate_q", "up_q", "down_q", "gate_s", "gate_b", "up_s", "up_b", "down_s",
                      "down_b")]
            assert np.array_equal(store[li, e], np.concatenate(parts))
