"""Query planning: tnb_batch_plan and first-hop query pruning, against the reference's outputs."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import load_golden
from minikg_dev_b200 import batching
from oracle import fastlog_oracle as O


@pytest.fixture(scope="module")
def pf():
    return load_golden("prune")


def _split(arr, off, i):
    return arr[off[i]:off[i + 1]]


class _Model:
    """The rule model surface ``prepare_rule_first_hop_prune`` reads."""

    def __init__(self, logits, tau, R, device="cpu"):
        self.logits = torch.from_numpy(logits)
        self.tau_1 = float(tau)
        self.relation_count = int(R)
        self.emb = torch.zeros(1, device=device)

    def build_rule_logits(self, rels):
        return self.logits[int(rels[0])][None].to(rels.device)


@pytest.mark.parametrize("dataset,nominal,expect", [
    ("family", 512, (512, 0)), ("wn18rr", 2048, (1024, 1024)), ("freebase", 512, (256, 256)),
    ("wn18rr", 5, (3, 2)), ("wn18rr", 3, (1, 2)), ("wn18rr", 1, (1, 0)), ("wn18rr", 0, (1, 0)),
    ("family", 0, (1, 0)), ("wn18rr", 2, (1, 1)), ("wn18rr", 7, (3, 4))])
def test_tnb_batch_plan(dataset, nominal, expect):
    plan = batching.tnb_batch_plan(SimpleNamespace(dataset=dataset), nominal)
    assert (plan.true_target_batch_size, plan.false_main_batch_count) == expect
    assert O.tnb_batch_plan(dataset, nominal) == expect


def test_oracle_first_hop_prune_vs_golden(pf):
    R = int(pf["pf_R"][0])
    rels = pf["pf_relations"]
    active = [_split(pf["pf_active"], pf["pf_active_off"], i) for i in range(len(rels))]
    for i, r in enumerate(rels):
        got = O.rule_first_hop_channels(pf["pf_logits"][r], pf["pf_tau"][0], pf["pf_threshold"][0])
        np.testing.assert_array_equal(got, active[i])
    wanted = sorted({int(c) % R for a in active for c in a if c < 2 * R})
    cache = O.rule_first_hop_cache(pf["pf_head"], pf["pf_rel"], pf["pf_tail"], pf["pf_supply"], wanted, R)
    assert sorted(cache) == pf["pf_cache_keys"].tolist()
    for j, c in enumerate(pf["pf_cache_keys"]):
        np.testing.assert_array_equal(cache[int(c)], _split(pf["pf_cache"], pf["pf_cache_off"], j))
    for i in range(len(rels)):
        q = _split(pf["pf_queries"], pf["pf_queries_off"], i)
        np.testing.assert_array_equal(O.rule_first_hop_query_heads(active[i], cache, q),
                                      _split(pf["pf_kept"], pf["pf_kept_off"], i))


def _run_prepare(pf, device):
    R = int(pf["pf_R"][0])
    model = _Model(pf["pf_logits"], pf["pf_tau"][0], R, device)
    facts = torch.from_numpy(np.stack([pf["pf_head"], pf["pf_rel"], pf["pf_tail"]], 1).astype(np.int64)).to(device)
    args = SimpleNamespace(decode_query_prune="rule_first_hop", decode_query_rule_threshold=float(pf["pf_threshold"][0]))
    batching.prepare_rule_first_hop_prune(model, pf["pf_relations"].tolist(), facts, pf["pf_supply"], args)
    return args


def _check_prepared(pf, args):
    rels = pf["pf_relations"]
    for i, r in enumerate(rels):
        assert args._decode_query_active_channels[int(r)] == _split(pf["pf_active"], pf["pf_active_off"], i).tolist()
        q = _split(pf["pf_queries"], pf["pf_queries_off"], i)
        got = batching.rule_first_hop_query_heads(int(r), q.tolist(), args)
        assert got == _split(pf["pf_kept"], pf["pf_kept_off"], i).tolist()
    assert sorted(args._decode_query_channel_heads) == pf["pf_cache_keys"].tolist()
    for j, c in enumerate(pf["pf_cache_keys"]):
        np.testing.assert_array_equal(args._decode_query_channel_heads[int(c)],
                                      _split(pf["pf_cache"], pf["pf_cache_off"], j))


def test_prepare_rule_first_hop_prune_host(pf):
    _check_prepared(pf, _run_prepare(pf, "cpu"))


def test_prune_disabled_paths(pf):
    model = _Model(pf["pf_logits"], pf["pf_tau"][0], int(pf["pf_R"][0]))
    facts = np.stack([pf["pf_head"], pf["pf_rel"], pf["pf_tail"]], 1)
    for args in (SimpleNamespace(decode_query_prune="none", decode_query_rule_threshold=0.2),
                 SimpleNamespace(decode_query_prune="rule_first_hop", decode_query_rule_threshold=0.0)):
        batching.prepare_rule_first_hop_prune(model, [0, 1], facts, pf["pf_supply"], args)
        assert not hasattr(args, "_decode_query_channel_heads")
        q = [5, 3, 5, 900 - 1]
        if args.decode_query_prune == "none":
            assert batching.rule_first_hop_query_heads(0, q, args) == q
        else:
            assert batching.rule_first_hop_query_heads(0, q, args) == []  # nothing prepared


def test_prune_empty_supply(pf):
    args = SimpleNamespace(decode_query_prune="rule_first_hop", decode_query_rule_threshold=0.2)
    model = _Model(pf["pf_logits"], pf["pf_tau"][0], int(pf["pf_R"][0]))
    facts = np.stack([pf["pf_head"], pf["pf_rel"], pf["pf_tail"]], 1)
    batching.prepare_rule_first_hop_prune(model, [0, 5], facts, np.zeros(len(facts), bool), args)
    assert all(v.size == 0 for v in args._decode_query_channel_heads.values())
    assert batching.rule_first_hop_query_heads(0, [1, 2, 3], args) == []


@pytest.mark.gpu
def test_prepare_rule_first_hop_prune_device(pf):
    _check_prepared(pf, _run_prepare(pf, "cuda"))


@pytest.mark.gpu
def test_first_hop_supported_entities_device_graph(pf):
    from minikg_dev_b200.graph import DeviceGraph
    E, R = int(pf["pf_E"][0]), int(pf["pf_R"][0])
    dev = torch.device("cuda")
    g = DeviceGraph.from_triples(torch.from_numpy(pf["pf_head"]).to(dev), torch.from_numpy(pf["pf_rel"]).to(dev),
                                 torch.from_numpy(pf["pf_tail"]).to(dev), E, R)
    supply = torch.from_numpy(pf["pf_supply"]).to(dev)
    for i in range(len(pf["pf_relations"])):
        chans = torch.from_numpy(_split(pf["pf_active"], pf["pf_active_off"], i))
        mask = batching.first_hop_supported_entities(g, chans, supply)
        q = torch.from_numpy(_split(pf["pf_queries"], pf["pf_queries_off"], i)).to(dev)
        kept = q[mask[q]].cpu().numpy()
        np.testing.assert_array_equal(kept, _split(pf["pf_kept"], pf["pf_kept_off"], i))
