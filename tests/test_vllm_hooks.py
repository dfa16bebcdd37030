"""The vLLM integration and DecodeView's host logic, on the CPU.

* ``require_supported_attention``: the refusals of the reference's own test (tests/test_supported_attention.py
  of the reference), with vLLM's own cache-spec classes and stand-in builders and layers.
* ``install_decode_view`` / ``install_audit_kernel``: each patches vLLM's Triton and FlashInfer classes once,
  and the patched methods hand the batch to the view, or record after the layer, as the reference's do
  (runtime/block_view.py:504-596). The original methods are stand-ins, restored after each test.
* ``attach_audit_plane``: the recording plane's table follows its layer names; another plane takes the runner's
  caches in order (:599-626).
* ``DecodeView``'s writes, releases and row reassignment, with its state on the CPU (``build`` needs the GPU).
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

pytest.importorskip("vllm")

from vllm.v1.attention.backend import AttentionType  # noqa: E402
from vllm.v1.kv_cache_interface import FullAttentionSpec, MambaSpec, SlidingWindowSpec  # noqa: E402

from ekv.runtime import block_view  # noqa: E402
from ekv.runtime.block_view import DecodeView, require_supported_attention  # noqa: E402

FULL = FullAttentionSpec(block_size=16, num_kv_heads=8, head_size=128, dtype=torch.float16)


def layer(sliding_window=None, alibi=None, attn_type=AttentionType.DECODER):
    return SimpleNamespace(sliding_window=sliding_window, impl=SimpleNamespace(alibi_slopes=alibi), attn_type=attn_type)


def builder(spec=FULL, layers=None, names=("l0", "l1"), rows=2):
    layers = layers or {name: layer() for name in names}
    return SimpleNamespace(
        kv_cache_spec=spec,
        layer_names=list(layers),
        vllm_config=SimpleNamespace(compilation_config=SimpleNamespace(static_forward_context=layers),
                                    scheduler_config=SimpleNamespace(max_num_seqs=rows)),
    )


@pytest.fixture
def fresh(monkeypatch):
    """No view or plane yet in this process, the compiler pass not asked for."""
    monkeypatch.setattr(block_view, "_view", None)
    monkeypatch.setattr(block_view, "_plane", None)
    monkeypatch.setattr(block_view, "_layers", ())
    monkeypatch.delenv("EKV_ATTN_SHARE", raising=False)
    monkeypatch.delenv("EKV_AUDIT_KERNEL", raising=False)
    monkeypatch.delenv("EKV_PREFILL_AUDIT", raising=False)


# ---- require_supported_attention -----------------------------------------------------------------------


def test_plain_full_attention_is_accepted():
    require_supported_attention(builder())


@pytest.mark.parametrize(
    "spec, match",
    [
        (SlidingWindowSpec(block_size=16, num_kv_heads=8, head_size=128, dtype=torch.float16, sliding_window=1024),
         "SlidingWindowSpec"),
        (MambaSpec(block_size=16, shapes=((1,),), dtypes=(torch.float16,)), "MambaSpec"),
        (FullAttentionSpec(block_size=16, num_kv_heads=8, head_size=128, dtype=torch.float16, sliding_window=512),
         "sliding window or chunked"),
        (FullAttentionSpec(block_size=16, num_kv_heads=8, head_size=128, dtype=torch.float16,
                           attention_chunk_size=256), "sliding window or chunked"),
    ],
)
def test_cache_groups_the_view_cannot_trim_are_refused(spec, match):
    with pytest.raises(RuntimeError, match=match):
        require_supported_attention(builder(spec))


@pytest.mark.parametrize(
    "bad, match",
    [(layer(sliding_window=4096), "layer bad has a sliding window"), (layer(alibi=torch.ones(8)), "position bias"),
     (layer(attn_type=AttentionType.ENCODER), "encoder")],
)
def test_layers_the_view_cannot_trim_are_refused_and_named(bad, match):
    with pytest.raises(RuntimeError, match=match):
        require_supported_attention(builder(layers={"ok": layer(), "bad": bad}))


def test_the_first_batch_makes_the_view_and_a_second_cache_group_is_refused(fresh):
    batch = SimpleNamespace(block_table_tensor=torch.zeros(3, 5, dtype=torch.int32))
    first, second = builder(names=("a", "b"), rows=3), builder(names=("c", "d"), rows=3)
    view = block_view._view_for(first, batch)
    assert (view.rows, view.width, view.block_size, view.audit) == (3, 5, 16, None)
    assert block_view._view_for(first, batch) is view and block_view.current_view() is view
    with pytest.raises(RuntimeError, match="several"):
        block_view._view_for(second, batch)


def test_the_compiler_pass_and_a_prefill_audit_are_refused(fresh, monkeypatch):
    batch = SimpleNamespace(block_table_tensor=torch.zeros(2, 4, dtype=torch.int32))
    monkeypatch.setenv("EKV_PREFILL_AUDIT", "1")
    with pytest.raises(RuntimeError, match="EKV_PREFILL_AUDIT"):
        block_view._view_for(builder(), batch)
    monkeypatch.delenv("EKV_PREFILL_AUDIT")
    monkeypatch.setenv("EKV_ATTN_SHARE", "1")
    with pytest.raises(RuntimeError, match="EKV_ATTN_SHARE"):
        block_view._view_for(builder(), batch)


def test_no_view_before_the_first_batch(fresh):
    with pytest.raises(RuntimeError, match="no attention batch"):
        block_view.current_view()


# ---- the patches -----------------------------------------------------------------------------------------


class FakeView:
    def __init__(self):
        self.calls = []
        self.table = torch.full((2, 4), 7, dtype=torch.int32)
        self.lens = torch.tensor([16, 32], dtype=torch.int32)
        self.audit = None

    def build(self, table, seq_lens, query_lens):
        self.calls.append(("build", query_lens.tolist()))
        return self.table, self.lens

    def skip(self, seq_lens, query_lens):
        self.calls.append(("skip", query_lens.tolist()))

    @property
    def buffers(self):
        return self.table, self.lens


def batch_metadata():
    """A CommonAttentionMetadata stand-in: two rows, one decoding and one prefilling 3 tokens."""

    class Batch(SimpleNamespace):
        def replace(self, **changes):
            return Batch(**{**vars(self), **changes})

    return Batch(block_table_tensor=torch.arange(8, dtype=torch.int32).view(2, 4),
                 seq_lens=torch.tensor([60, 30], dtype=torch.int32),
                 query_start_loc_cpu=torch.tensor([0, 1, 4], dtype=torch.int32), num_reqs=2)


@pytest.fixture
def stub_backends(monkeypatch):
    """vLLM's builders and implementations with stand-in originals that record what they were given."""
    from vllm.v1.attention.backends.flashinfer import FlashInferImpl, FlashInferMetadataBuilder
    from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl, TritonAttentionMetadataBuilder

    seen = []

    def original_build(self, common_prefix_len, common_attn_metadata, fast_build=False):
        seen.append(("original", common_prefix_len, common_attn_metadata))
        return SimpleNamespace(block_table=None, seq_lens=None)

    def original_forward(self, layer, query, key, value, kv_cache, attn_metadata, *args, **kwargs):
        seen.append(("forward", layer.layer_name))
        return "output"

    for cls in (TritonAttentionMetadataBuilder, FlashInferMetadataBuilder):
        monkeypatch.setattr(cls, "build", original_build)
    for cls in (TritonAttentionImpl, FlashInferImpl):
        monkeypatch.setattr(cls, "forward", original_forward)
    return seen


def test_install_decode_view_patches_each_builder_once(stub_backends):
    from vllm.v1.attention.backends.flashinfer import FlashInferMetadataBuilder
    from vllm.v1.attention.backends.triton_attn import TritonAttentionMetadataBuilder

    assert block_view.install_decode_view() == 2
    assert block_view.install_decode_view() == 0  # already patched
    assert TritonAttentionMetadataBuilder.build._ekv_decode_view and FlashInferMetadataBuilder.build._ekv_decode_view


def test_the_triton_builder_gets_the_views_buffers(stub_backends, monkeypatch):
    from vllm.v1.attention.backends.triton_attn import TritonAttentionMetadataBuilder

    view = FakeView()
    monkeypatch.setattr(block_view, "_view_for", lambda builder, batch: view)
    block_view.install_decode_view()
    metadata = TritonAttentionMetadataBuilder.build(object(), 0, batch_metadata())
    assert metadata.block_table is view.table and metadata.seq_lens is view.lens
    assert view.calls == [("build", [1, 3])]
    metadata = TritonAttentionMetadataBuilder.build(object(), 5, batch_metadata())  # a shared-prefix cascade
    assert metadata.block_table is None and view.calls[-1] == ("skip", [1, 3])


def test_the_flashinfer_builder_plans_from_the_view(stub_backends, monkeypatch):
    from vllm.v1.attention.backends.flashinfer import FlashInferMetadataBuilder

    view = FakeView()
    monkeypatch.setattr(block_view, "_view_for", lambda builder, batch: view)
    block_view.install_decode_view()
    FlashInferMetadataBuilder.build(object(), 0, batch_metadata())
    _, prefix, given = stub_backends[-1]
    assert prefix == 0 and given.block_table_tensor is view.table and given.seq_lens is view.lens
    assert given.max_seq_len == 32 and given._seq_lens_cpu is None
    FlashInferMetadataBuilder.build(object(), 3, batch_metadata())
    _, prefix, given = stub_backends[-1]
    assert prefix == 3 and given.block_table_tensor.tolist() == batch_metadata().block_table_tensor.tolist()
    assert view.calls == [("build", [1, 3]), ("skip", [1, 3])]


def test_install_audit_kernel_records_after_each_attention_layer(stub_backends, monkeypatch):
    from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl

    from ekv.runtime.audit_kernel import RecordingPlane

    class Plane(RecordingPlane):
        def __init__(self):  # no device state: only record() is called
            self.recorded = []

        def record(self, layer_name, table, lens, query, kv_cache, scale):
            self.recorded.append((layer_name, table, lens, query, kv_cache, scale))

    view = FakeView()
    view.audit = Plane()
    monkeypatch.setattr(block_view, "_view", view)
    assert block_view.install_audit_kernel() == 2
    assert block_view.install_audit_kernel() == 0
    impl = SimpleNamespace(scale=0.125)
    q, kv = torch.zeros(2, 4, 8), torch.zeros(3, 2, 16, 1, 8)
    out = TritonAttentionImpl.forward(impl, SimpleNamespace(layer_name="model.layers.0.attn"), q, None, None, kv,
                                      object())
    assert out == "output" and stub_backends[-1] == ("forward", "model.layers.0.attn")
    name, table, lens, query, cache, scale = view.audit.recorded[-1]
    assert name == "model.layers.0.attn" and table is view.table and lens is view.lens
    assert query is q and cache is kv and scale == 0.125
    TritonAttentionImpl.forward(impl, SimpleNamespace(layer_name="x"), q, None, None, kv, None)  # a profiling run
    assert len(view.audit.recorded) == 1
    view.audit = None
    with pytest.raises(RuntimeError, match="no recording plane"):
        TritonAttentionImpl.forward(impl, SimpleNamespace(layer_name="y"), q, None, None, kv, object())


def test_attach_audit_plane_fills_the_layer_table(monkeypatch):
    from ekv.runtime.audit_kernel import RecordingPlane

    class Recording(RecordingPlane):
        def __init__(self):
            self.attached = None

        @property
        def layer_names(self):
            return ["b", "a"]

        def attach(self, addresses):
            self.attached = addresses
            return True

    class Other:
        attached = None

        def attach(self, addresses):
            self.attached = addresses
            return True

    caches = {name: SimpleNamespace(kv_cache=torch.zeros(4) + i) for i, name in enumerate("ab")}
    runner = SimpleNamespace(compilation_config=SimpleNamespace(static_forward_context=caches),
                             kv_caches=[caches["a"].kv_cache, None, caches["b"].kv_cache])
    view = object()
    monkeypatch.setattr(block_view, "_view", view)
    plane = Recording()
    monkeypatch.setattr(block_view, "_plane", plane)
    assert block_view.attach_audit_plane(runner) is view
    assert plane.attached == [caches["b"].kv_cache.data_ptr(), caches["a"].kv_cache.data_ptr()]
    other = Other()
    monkeypatch.setattr(block_view, "_plane", other)
    block_view.attach_audit_plane(runner)
    assert other.attached == [caches["a"].kv_cache.data_ptr(), caches["b"].kv_cache.data_ptr()]


# ---- DecodeView's host logic -------------------------------------------------------------------------


class Switch:
    def set(self, on):
        pass

    def select(self, audited, token_start):
        pass


def cpu_view(**kwargs):
    return DecodeView(rows=3, width=4, block_size=16, device=torch.device("cpu"), **kwargs)


def test_writes_are_validated_and_kept_in_the_views_state():
    view = cpu_view()
    assert view.keep.all() and not view.released.any()
    mask = np.array([[1, 0, 0, 1], [1, 1, 0, 0], [0, 0, 0, 0]], dtype=np.uint32)
    assert view.write_row_controls(mask) == 1 and view.version == 1
    np.testing.assert_array_equal(view.keep, mask != 0)
    with pytest.raises(ValueError):
        view.write_row_controls(mask, np.zeros((3, 4), dtype=np.float32))
    with pytest.raises(ValueError):
        view.write_row_controls(np.ones((2, 4)))
    with pytest.raises(ValueError):
        view.write_audit_rows(np.array([True, False, False]))  # no plane to switch the statistic on
    with pytest.raises(ValueError):
        DecodeView(rows=2, width=4, block_size=16, prefill_audit=True, device=torch.device("cpu"))
    view.write_final_prefill(np.array([False, True]))
    assert view.final_prefill.tolist() == [False, True, False]
    with pytest.raises(RuntimeError, match="CUDA"):
        view.build(torch.zeros(3, 4, dtype=torch.int32), torch.zeros(3, dtype=torch.int32), torch.ones(3))


def test_release_needs_a_covering_audit_and_keeps_block_zero_and_the_last_block():
    view = cpu_view(audit=Switch())
    ask = np.ones((3, 4), dtype=np.uint8)
    assert view.write_release(ask) == []  # no audit yet
    view.row_audited[0], view.audited_blocks[0] = True, 4
    view.row_audited[2], view.audited_blocks[2] = True, 1
    assert view.write_release(ask) == [(0, 1), (0, 2)]
    assert view.write_release(ask) == []  # released once
    assert view.released[0].tolist() == [False, True, True, False] and not view.released[1:].any()


def test_reassigned_rows_carry_their_state_and_new_rows_start_fresh():
    view = cpu_view(audit=Switch())
    view.write_row_controls(np.array([[1, 0, 0, 1], [1, 1, 0, 0], [0, 1, 0, 1]]))
    view.row_audited[0], view.audited_blocks[0] = True, 4
    view.write_release(np.array([[0, 1, 0, 0], [0, 0, 0, 0], [0, 0, 0, 0]]))
    view.write_audit_rows(np.array([False, True, False]))
    view.reassign_rows({1: 0, 0: 1}, [2], [])  # rows 0 and 1 swap requests; row 2 holds a new one
    assert view.keep.tolist() == [[1, 1, 0, 0], [1, 0, 0, 1], [1, 1, 1, 1]]
    assert view.released[1].tolist() == [False, True, False, False] and not view.released[[0, 2]].any()
    assert view.row_audited.tolist() == [False, True, False] and view.audited_blocks.tolist() == [0, 4, 0]
    assert view.audit_rows.tolist() == [True, False, True]  # the moved request and the new one (first decode)
    view.reassign_rows({}, [], [1])  # row 1 now holds nothing
    assert view.keep[1].all() and not view.released[1].any() and not view.row_audited[1]
    assert view.audit_rows.tolist() == [True, False, True] and view.version == 3  # a commit, two reassignments
