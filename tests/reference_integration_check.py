"""INTEGRATION.md section 2, executed against the reference's own engine (run by
``tests/test_reference_integration_cpu.py`` in a subprocess; needs the reference's source tree).

1. ``import rocketllm_b200.quant`` (the package's transformers quantizer and experts function),
   then the reference's ``register_backend(RW4Backend)``; the reference's ``detect_backend`` must
   return the RW4 backend for ``quant_method: rw4`` (``rocketllm/quant/registry.py:656-675``).
2. The reference's ``RocketModel(path, device="cpu", dtype=torch.bfloat16)`` on a 2-layer RW4
   checkpoint: its ``init_model`` runs the package's quantizer (``rocketllm/base.py:680-703``), so
   the model's Linear layers are ``RW4Linear`` modules; its ``load_layer_to_cpu`` +
   ``move_layer_to_device`` (``rocketllm/base.py:836-950``) place every layer through
   ``_move_coalesced`` (``:952-991``) with the RW4 backend's plan: the packed triples must land
   verbatim (uint8 codes, fp16 scales and zeros, bit-identical to the checkpoint) as views of one
   coalesced buffer per dtype, and the norms in the compute dtype.
Prints ``ok`` on success.  The forward itself needs a GPU (``RW4Linear`` has no CPU path), which is
what ``tests/test_tinyllama_gpu.py`` runs on the package's own engine.
"""
import os
import sys
import tempfile

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(HERE, "golden"))


def main():
    import reference_harness as rh
    rocketllm = rh.import_reference()
    import rocketllm_b200.quant  # noqa: F401 - registers the package's rw4 quantizer
    from oracle import rw4_oracle as o
    from rocketllm.quant import detect_backend, register_backend
    from rocketllm_b200.quant import RW4Backend, RW4Linear
    from rocketllm_b200.synthetic import TINYLLAMA, write_rw4_llama

    register_backend(RW4Backend)
    backend = detect_backend({"quant_method": "rw4", "bits": 4, "group_size": 64})
    assert isinstance(backend, RW4Backend), type(backend)
    assert not backend.needs_scratch(None)

    def oracle_quantize(w):
        packed, scale, zero, _ = o.quantize(w.numpy(), 64, "f32")
        return torch.from_numpy(packed), torch.from_numpy(scale), torch.from_numpy(zero)

    class TokenIdModel(rocketllm.base.RocketModel):
        def get_tokenizer(self, hf_token=None):
            return None

    cfg = dict(TINYLLAMA, num_hidden_layers=2, hidden_size=256, intermediate_size=512,
               num_attention_heads=4, num_key_value_heads=2, head_dim=64, vocab_size=512)
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "rw4")
        sd = write_rw4_llama(path, cfg, oracle_quantize)
        model = TokenIdModel(path, device="cpu", dtype=torch.bfloat16)
        assert isinstance(model.quant, RW4Backend), type(model.quant)
        layer = model.model.model.layers[0]
        assert isinstance(layer.self_attn.q_proj, RW4Linear)
        for i in range(cfg["num_hidden_layers"]):
            name = f"model.layers.{i}"
            moved = model.move_layer_to_device(model.load_layer_to_cpu(name))
            prefix = name + "."
            assert len(moved) == sum(1 for k in sd if k.startswith(prefix)), moved
            storages = set()
            for key, want in sd.items():
                if not key.startswith(prefix):
                    continue
                got = model.model.get_parameter(key)
                if key.endswith(("_packed", "_scale", "_zero_point")):
                    assert got.dtype == want.dtype, (key, got.dtype)
                    assert torch.equal(got.view(torch.uint8), want.view(torch.uint8)), key
                    storages.add((got.dtype, got.untyped_storage().data_ptr()))
                else:
                    assert got.dtype == torch.bfloat16, (key, got.dtype)
                    assert torch.equal(got, want.to(torch.bfloat16)), key
            # one coalesced buffer per target dtype (uint8 codes, fp16 scales and zeros)
            assert len({s for s in storages}) == len({d for d, _ in storages}), storages
    print("ok")


if __name__ == "__main__":
    main()
