"""Which linear -> all_reduce -> add chains of a plan run as one fused kernel (CPU).

``CudaBackend._allreduce_fusions`` is plan logic: at TP > 1 with
``allreduce="fused"`` every decode o_proj / down_proj chain qualifies; a command
between the linear and the add that touches the add's output, or writes its
residual, disqualifies the chain; row batches (prefill) and the other modes never
fuse.  Run here on a stand-in HAL object (no GPU).
"""

from __future__ import annotations

import types
from dataclasses import replace

import pytest

from backend import hal_cuda
from contracts.exec_plan import Access, Command


class _Group:
    size = 2

    @staticmethod
    def fits(nbytes: int) -> bool:
        return nbytes % 16 == 0 and 0 < nbytes <= 256 << 10


def _hal(plan, mode="fused", size=2):
    import torch

    g = _Group()
    g.size = size
    return types.SimpleNamespace(_p2p=g, local=[0], config=types.SimpleNamespace(allreduce=mode),
                                 _host={id(plan): torch.zeros(plan.meta["host_layout"].total, dtype=torch.uint8)})


def _plan(phase="decode", tp=2, layers=2, prompt=16):
    from graph.llama import ModelConfig
    from runtime.program import compile_llama

    prog = compile_llama(ModelConfig.llama2_7b(max_seq=64, num_layers=layers), tp, batch=1, prompt_len=prompt)
    return prog.plans[phase]


def _fusions(plan, **kw):
    return hal_cuda.CudaBackend._allreduce_fusions(_hal(plan, **kw), plan)


def test_every_decode_chain_fuses_and_its_sum_needs_no_write():
    plan = _plan()
    f = _fusions(plan)
    nodes = sorted((v[0].payload["node"], v[2].payload["node"]) for v in f.values())
    assert nodes == [("l0.down_proj", "l0.resid_mlp"), ("l0.o_proj", "l0.resid_attn"),
                     ("l1.down_proj", "l1.resid_mlp"), ("l1.o_proj", "l1.resid_attn")]
    for lin, comb, add, sum_in_add, sum_out in f.values():
        assert comb.payload["kind"] == "all_reduce"
        assert any(r[0] == sum_in_add for r in add.payload["inputs"])
        assert sum_out is None  # only the add reads the all-reduced sum


@pytest.mark.parametrize("mode", ["ordered", "p2p", "nccl"])
def test_only_the_fused_mode_fuses(mode):
    assert _fusions(_plan(), mode=mode) == {}


def test_row_batches_do_not_fuse():
    assert _fusions(_plan("prefill")) == {}


def test_a_reader_of_the_add_output_between_linear_and_add_blocks_the_chain():
    plan = _plan(layers=1)
    (lin, comb, add, _, _), = [v for v in _fusions(plan).values() if v[0].payload["node"] == "l0.o_proj"]
    y = add.payload["output"]
    spy = Command(id=10 ** 6, op="launch", dpu_id=0, payload={"kernel": "materialize", "node": "spy"},
                  reads=[Access(("dpu", 0), y[0], 16)])
    cmds = list(plan.commands)
    cmds.insert(cmds.index(comb), spy)
    blocked = replace(plan, commands=cmds)
    nodes = {v[0].payload["node"] for v in _fusions(blocked).values()}
    assert "l0.o_proj" not in nodes and "l0.down_proj" in nodes


def test_a_writer_of_the_residual_between_linear_and_add_blocks_the_chain():
    plan = _plan(layers=1)
    (lin, comb, add, sum_in_add, _), = [v for v in _fusions(plan).values() if v[0].payload["node"] == "l0.down_proj"]
    res = next(r for r in add.payload["inputs"] if r[0] != sum_in_add)
    spy = Command(id=10 ** 6, op="launch", dpu_id=0, payload={"kernel": "materialize", "node": "spy"},
                  writes=[Access(("dpu", 0), res[0], 16)])
    cmds = list(plan.commands)
    cmds.insert(cmds.index(comb), spy)
    nodes = {v[0].payload["node"] for v in _fusions(replace(plan, commands=cmds)).values()}
    assert "l0.down_proj" not in nodes and "l0.o_proj" in nodes


def test_a_later_reader_of_the_sum_makes_the_kernel_write_it():
    plan = _plan(layers=1)
    (lin, comb, add, sum_in_add, _), = [v for v in _fusions(plan).values() if v[0].payload["node"] == "l0.o_proj"]
    nbytes = comb.payload["entry"].numel * comb.payload["entry"].dtype.itemsize
    spy = Command(id=10 ** 6, op="launch", dpu_id=0, payload={"kernel": "materialize", "node": "spy"},
                  reads=[Access(("dpu", 0), sum_in_add, nbytes)])
    cmds = list(plan.commands)
    cmds.insert(cmds.index(add) + 1, spy)
    f = {v[0].payload["node"]: v for v in _fusions(replace(plan, commands=cmds)).values()}
    assert f["l0.o_proj"][4] == sum_in_add


# ---- combine + add (allreduce="ordered", combine_add) ------------------------------


def _hal_ordered(plan, combine_add=True, split=0, tp=2):
    import torch

    cfg = types.SimpleNamespace(allreduce="ordered", combine_add=combine_add, num_dpus=tp,
                                allreduce_split_bytes=split)
    return types.SimpleNamespace(distributed=True, local=[0], config=cfg,
                                 _host={id(plan): torch.zeros(plan.meta["host_layout"].total, dtype=torch.uint8)})


def _comb_add(plan, **kw):
    return hal_cuda.CudaBackend._combine_add_fusions(_hal_ordered(plan, **kw), plan)


def test_every_decode_all_reduce_folds_its_add_into_the_combine():
    plan = _plan()
    f = _comb_add(plan)
    adds = sorted(v[0].payload["node"] for v in f.values())
    assert adds == ["l0.resid_attn", "l0.resid_mlp", "l1.resid_attn", "l1.resid_mlp"]
    for cid, (add, res_off, y_off, sum_off) in f.items():
        comb = plan.commands[cid]
        assert comb.payload["kind"] == "all_reduce"
        assert add.payload["output"][0] == y_off and any(r[0] == res_off for r in add.payload["inputs"])
        assert sum_off is None


def test_combine_add_is_off_unless_asked_and_respects_the_split_threshold():
    plan = _plan()
    assert _comb_add(plan, combine_add=False) == {}
    assert _comb_add(plan, split=8192) == {}  # 4096 bf16 = 8 KB edges take the split path
    assert len(_comb_add(plan, split=8193)) == 4


def test_a_reader_of_the_add_output_between_combine_and_add_blocks_the_fold():
    plan = _plan(layers=1)
    f = _comb_add(plan)
    cid, (add, _, y_off, _) = next((k, v) for k, v in f.items() if v[0].payload["node"] == "l0.resid_attn")
    spy = Command(id=10 ** 6, op="launch", dpu_id=0, payload={"kernel": "materialize", "node": "spy"},
                  reads=[Access(("dpu", 0), y_off, 16)])
    cmds = list(plan.commands)
    cmds.insert(cmds.index(add), spy)
    nodes = {v[0].payload["node"] for v in _comb_add(replace(plan, commands=cmds)).values()}
    assert "l0.resid_attn" not in nodes and "l0.resid_mlp" in nodes


def test_a_later_reader_of_the_sum_makes_the_fold_write_it():
    plan = _plan(layers=1)
    f = _comb_add(plan)
    cid, (add, _, _, _) = next((k, v) for k, v in f.items() if v[0].payload["node"] == "l0.resid_mlp")
    comb = plan.commands[cid]
    wb = [s for s in comb.payload["entry"].writeback_segments if s.dst_dpu == 0][0]
    spy = Command(id=10 ** 6, op="launch", dpu_id=0, payload={"kernel": "materialize", "node": "spy"},
                  reads=[Access(("dpu", 0), wb.dst_addr, wb.nbytes)])
    cmds = list(plan.commands)
    cmds.insert(cmds.index(add) + 1, spy)
    g = {v[0].payload["node"]: v for v in _comb_add(replace(plan, commands=cmds)).values()}
    assert g["l0.resid_mlp"][3] == wb.dst_addr


def test_prefill_row_batches_fold_too():
    """Unlike the fused projection kernel, the combine fold has no row limit."""
    plan = _plan("prefill")
    assert len(_comb_add(plan)) == 4


# ---- decode attention inside attn_in (fuse_attention) ---------------------------------


def _hal_attn(plan, ranks=(0,), on=True):
    cfg = types.SimpleNamespace(fuse_attention=on)
    return types.SimpleNamespace(config=cfg, _arena={r: None for r in ranks})


def _attn(plan, **kw):
    return hal_cuda.CudaBackend._attention_fusions(_hal_attn(plan, **kw), plan)


@pytest.mark.parametrize("tp", [1, 2])
def test_every_decode_attention_folds_into_its_attn_in(tp):
    plan = _plan(tp=tp)
    f = _attn(plan, ranks=tuple(range(tp)))
    assert len(f) == 2 * tp  # 2 layers x ranks
    by_id = {c.id: c for c in plan.commands}
    for ai_id, att in f.items():
        ai = by_id[ai_id]
        assert ai.payload["kernel"] == "attn_in" and att.payload["kernel"] == "attention"
        assert ai.dpu_id == att.dpu_id and ai.payload["output"][0] == att.payload["inputs"][0][0]
        assert ai.payload["node"].split(".")[0] == att.payload["node"].split(".")[0]  # same layer


def test_attention_fold_is_off_unless_asked_and_only_for_decode_rows():
    assert _attn(_plan(), on=False) == {}
    assert _attn(_plan("prefill")) == {}  # 16 prompt rows: the row-batch kernels


def test_a_reader_of_the_attention_output_before_the_attention_blocks_the_fold():
    plan = _plan(tp=1, layers=1)
    (ai_id, att), = _attn(plan).items()
    out = att.payload["output"][0]
    spy = Command(id=10 ** 6, op="launch", dpu_id=0, payload={"kernel": "materialize", "node": "spy"},
                  reads=[Access(("dpu", 0), out, 16)])
    cmds = list(plan.commands)
    cmds.insert(cmds.index(att), spy)
    assert _attn(replace(plan, commands=cmds)) == {}


def test_a_writer_of_the_kv_before_the_attention_blocks_the_fold():
    plan = _plan(tp=1, layers=1)
    (ai_id, att), = _attn(plan).items()
    ai = next(c for c in plan.commands if c.id == ai_id)
    kv = next(a for a in ai.writes if a.offset != ai.payload["output"][0])
    spy = Command(id=10 ** 6, op="launch", dpu_id=0, payload={"kernel": "materialize", "node": "spy"},
                  writes=[Access(("dpu", 0), kv.offset + 64, 16)])
    cmds = list(plan.commands)
    cmds.insert(cmds.index(att), spy)
    assert _attn(replace(plan, commands=cmds)) == {}


def test_an_attention_output_over_the_attn_in_input_blocks_the_fold():
    # the fused launch writes the first heads while other CTAs still read the layer input
    plan = _plan(tp=1, layers=1)
    (ai_id, att), = _attn(plan).items()
    ai = next(c for c in plan.commands if c.id == ai_id)
    x = ai.payload["inputs"][0][0]
    moved = replace(att, payload={**att.payload, "output": (x,) + tuple(att.payload["output"][1:])})
    cmds = [moved if c is att else c for c in plan.commands]
    assert _attn(replace(plan, commands=cmds)) == {}


# ---- one launch per decode layer (decode_layer) --------------------------------------


def _hal_layer(tp=1, on=True, distributed=False, rank=0, step=False):
    cfg = types.SimpleNamespace(decode_layer=on, num_dpus=tp, decode_step=step)
    return types.SimpleNamespace(config=cfg, distributed=distributed, local=[rank], _arena={rank: None})


def _layers(plan, fused=None, **kw):
    return hal_cuda.CudaBackend._decode_layer_fusions(_hal_layer(**kw), plan, fused)


def test_every_decode_layer_runs_as_one_launch_at_tp1():
    plan = _plan(tp=1)
    f = _layers(plan)
    assert len(f) == 2
    for ai_id, (chain, ar) in f.items():
        assert chain[0].id == ai_id and ar is None
        assert [c.payload["kernel"] for c in chain] == ["attn_in", "attention", "linear_add", "mlp_in", "linear_add"]
        layer = chain[0].payload["node"].split(".")[0]
        assert all(c.payload["node"].split(".")[0] == layer for c in chain)
        for prev, nxt in zip(chain, chain[1:]):
            assert nxt.payload["inputs"][0][0] == prev.payload["output"][0]


def test_decode_layer_is_off_unless_asked_and_only_for_one_decode_row_at_tp1():
    assert _layers(_plan(tp=1), on=False) == {}
    assert _layers(_plan("prefill", tp=1)) == {}
    assert _layers(_plan(tp=2), tp=2) == {}
    assert _layers(_plan(tp=1), distributed=True) == {}


def test_a_command_inside_the_layer_breaks_the_chain():
    plan = _plan(tp=1, layers=1)
    (ai_id, (chain, _)), = _layers(plan).items()
    spy = Command(id=10 ** 6, op="launch", dpu_id=0, payload={"kernel": "materialize", "node": "spy"})
    cmds = list(plan.commands)
    cmds.insert(cmds.index(chain[3]), spy)
    assert _layers(replace(plan, commands=cmds)) == {}


def test_a_layer_whose_attention_output_overlaps_the_input_is_not_fused():
    plan = _plan(tp=1, layers=1)
    (ai_id, (chain, _)), = _layers(plan).items()
    att, o = chain[1], chain[2]
    x = chain[0].payload["inputs"][0][0]
    moved_att = replace(att, payload={**att.payload, "output": (x,) + tuple(att.payload["output"][1:])})
    moved_o = replace(o, payload={**o.payload, "inputs": [(x,) + tuple(o.payload["inputs"][0][1:])]
                                  + list(o.payload["inputs"][1:])})
    cmds = [moved_att if c is att else moved_o if c is o else c for c in plan.commands]
    assert _layers(replace(plan, commands=cmds)) == {}


@pytest.mark.parametrize("rank", [0, 1])
def test_at_tp2_fused_mode_each_layer_with_its_two_all_reduces_is_one_launch(rank):
    plan = _plan(tp=2)
    fused = hal_cuda.CudaBackend._allreduce_fusions(_hal(plan), plan) if rank == 0 else None
    if rank == 1:  # the same chains seen from rank 1's process
        h = _hal(plan)
        h.local = [1]
        fused = hal_cuda.CudaBackend._allreduce_fusions(h, plan)
    assert len(fused) == 4
    f = _layers(plan, fused, tp=2, distributed=True, rank=rank)
    assert len(f) == 2
    for ai_id, (chain, (o_chain, d_chain)) in f.items():
        assert [c.payload["kernel"] for c in chain] == ["attn_in", "attention", "linear", "mlp_in", "linear"]
        assert all(int(c.dpu_id) == rank for c in chain)
        assert o_chain[0] is chain[2] and d_chain[0] is chain[4]
        assert chain[3].payload["inputs"][0][0] == o_chain[2].payload["output"][0]  # mlp_in reads the add
        assert [c.payload["node"].split(".")[1] for c in chain] == ["q_rot", "attn", "o_proj", "mlp_act",
                                                                     "down_proj"]


def test_at_tp2_the_layer_needs_the_fused_mode_and_one_process_per_gpu():
    plan = _plan(tp=2)
    fused = hal_cuda.CudaBackend._allreduce_fusions(_hal(plan), plan)
    assert _layers(plan, {}, tp=2, distributed=True) == {}  # other all-reduce modes
    assert _layers(plan, fused, tp=2, distributed=False) == {}  # one process, several ranks
    assert _layers(plan, fused, tp=2, distributed=True, on=False) == {}


def _steps(plan, fused=None, **kw):
    h = _hal_layer(step=True, **kw)
    layers = hal_cuda.CudaBackend._decode_layer_fusions(h, plan, fused)
    return hal_cuda.CudaBackend._decode_step_fusion(h, plan, fused, layers)


def test_at_tp1_the_whole_decode_step_is_one_launch():
    plan = _plan(tp=1)
    (first, (run, head)), = _steps(plan).items()
    assert [chain[0].payload["node"] for chain, _ in run] == ["l0.q_rot", "l1.q_rot"]
    assert run[0][0][0].id == first and head.payload["kernel"] == "lm_head_in"
    assert head.payload["inputs"][0][0] == run[-1][0][4].payload["output"][0]
    assert _steps(_plan("prefill", tp=1)) == {}


@pytest.mark.parametrize("rank", [0, 1])
def test_at_tp2_fused_mode_the_whole_decode_step_is_one_launch_per_rank(rank):
    plan = _plan(tp=2)
    h = _hal(plan)
    h.local = [rank]
    fused = hal_cuda.CudaBackend._allreduce_fusions(h, plan)
    (first, (run, head)), = _steps(plan, fused, tp=2, distributed=True, rank=rank).items()
    assert len(run) == 2 and all(ar is not None for _, ar in run)
    assert int(head.dpu_id) == rank
    assert head.payload["inputs"][0][0] == run[-1][1][1][2].payload["output"][0]  # the last add's output


def test_a_command_between_the_last_layer_and_the_head_keeps_the_layers_apart():
    plan = _plan(tp=1)
    cmds = list(plan.commands)
    head = next(c for c in cmds if c.payload.get("kernel") == "lm_head_in")
    spy = Command(id=10 ** 6, op="launch", dpu_id=0, payload={"kernel": "materialize", "node": "spy"})
    cmds.insert(cmds.index(head), spy)
    blocked = replace(plan, commands=cmds)
    assert _steps(blocked) == {}
    assert len(_layers(blocked)) == 2  # each layer still fuses on its own



# ---- the arguments the HAL builds for the layer and step kernels pass the library's checks


class _FakeGroup(_Group):
    @staticmethod
    def descriptor(err):
        return 0x7000_0000


def _lowering_hal():
    return types.SimpleNamespace(arena_ptr=lambda r: 1 << 32, stream_handle=lambda r: 0,
                                 error_flag_ptr=lambda r: 1 << 24, scratch=lambda r, n, pool=None: (1 << 28, n),
                                 _p2p=_FakeGroup())


@pytest.mark.parametrize("tp", [1, 2])
def test_hal_built_layer_and_step_arguments_pass_the_library_checks(tp):
    """Every check of pim_decode_layer / pim_decode_step_prepare passes on the arguments
    lowered from the plan; the calls stop at the (deliberately absent) barrier or table,
    before any device work."""
    import ctypes

    from backend import _native as nat
    from backend.cuda_kernels import _layer_args, projection_args

    plan = _plan(tp=tp)
    kw = dict(tp=tp, distributed=tp > 1)
    fused = None
    if tp > 1:
        fused = hal_cuda.CudaBackend._allreduce_fusions(_hal(plan), plan)
    (first, (run, head)), = _steps(plan, fused, **kw).items()
    fake = _lowering_hal()
    every = []
    for chain, ar in run:
        args = _layer_args(fake, 0, chain, ar)
        assert (args[1].p2p_desc is not None) == (tp > 1)
        rc = nat.lib.pim_decode_layer(*[ctypes.byref(a) for a in args], None, None, nat.BF16, None)
        assert rc == 1 and b"null barrier" in nat.lib.pim_last_error(), nat.lib.pim_last_error()
        every += args
    head_args = projection_args(fake, 0, head)[0]
    ptrs = (ctypes.POINTER(nat.ProjectionArgs) * len(every))(*[ctypes.pointer(a) for a in every])
    out = ctypes.c_void_p()
    rc = nat.lib.pim_decode_step_prepare(ptrs, len(run), ctypes.byref(head_args), nat.BF16, None, 0,
                                         ctypes.byref(out))
    assert rc == 1 and b"table too small" in nat.lib.pim_last_error(), nat.lib.pim_last_error()
    assert not out.value


def test_decode_step_alone_implies_the_layer_fusions():
    plan = _plan(tp=1)
    h = _hal_layer(on=False, step=True)
    layers = hal_cuda.CudaBackend._decode_layer_fusions(h, plan, None)
    assert len(layers) == 2
    assert len(hal_cuda.CudaBackend._decode_step_fusion(h, plan, None, layers)) == 1
