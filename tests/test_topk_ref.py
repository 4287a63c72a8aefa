"""CPU checks of the second restatement of router_topk.comp (oracle/router_topk_ref.py) against
the vectorised oracle's routing (moe_oracle.softmax_f32 + topk_desc) and against hand-made cases:
exact ties go to the lower expert index, a later equal probability never displaces an earlier
one, and the shared entry's id 0 is mapped to the library's id E."""
import numpy as np

import moe_oracle as O
import router_topk_ref as R


def test_matches_vectorised_oracle_on_random_logits():
    rng = np.random.default_rng(5)
    for t in range(12):
        lg = (rng.normal(0, 1, 256) * (0.5 + t)).astype(np.float32)
        ent = R.route_token(lg)
        ids, w = O.topk_desc(O.softmax_f32(lg[None]), 8)
        assert [e for e, _ in ent[1:]] == ids[0].tolist()
        assert np.allclose([v for _, v in ent[1:]], w[0], rtol=2e-6, atol=0)
        assert ent[0] == (0, np.float32(1.0))


def test_exact_ties_keep_index_order():
    lg = np.full(256, -5.0, np.float32)
    lg[[200, 17, 3, 99]] = 2.0     # four equal maxima
    lg[[250, 251]] = 1.5
    lg[[10, 11, 12]] = 1.0         # three equal values compete for the last two slots
    ent = R.route_token(lg)
    assert [e for e, _ in ent[1:]] == [3, 17, 99, 200, 250, 251, 10, 11]
    ids, _ = O.topk_desc(O.softmax_f32(lg[None]), 8)
    assert ids[0].tolist() == [3, 17, 99, 200, 250, 251, 10, 11]


def test_shared_entry_mapping():
    lg = np.zeros(256, np.float32)
    lg[0] = 3.0  # routed expert 0 wins slot 1 while the reference's shared entry also says id 0
    ent = R.route_token(lg)
    assert ent[0][0] == 0 and ent[1][0] == 0
    lib = R.to_library_record(ent, 256, 0.25)
    assert lib[0] == (256, np.float32(0.25)) and lib[1][0] == 0
