"""Config-5 path on the GPU: the synthetic Gemma-4-shaped decoder with
attention routed through register_triton_attention() ("triton_gqa") against
the same model with explicit fp32 attention, in the spirit of the reference's
integration test (cosine of logits > 0.999 and top-1 agreement)."""
import pytest
import torch

pytest.importorskip("transformers")
from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS  # noqa: E402

from gemma_triton_flash_attn import register_triton_attention  # noqa: E402
from gemma_triton_flash_attn.gemma4_synthetic import Gemma4SyntheticConfig, Gemma4SyntheticDecoder  # noqa: E402
from test_decoder_cpu import explicit_attention  # noqa: E402

pytestmark = pytest.mark.gpu


def cfg(impl):
    # Real head dims (512 global, 256 sliding), reduced width and depth.
    return Gemma4SyntheticConfig(vocab_size=2000, hidden_size=512, num_layers=5, global_heads=8, global_kv_heads=1,
                                 global_head_dim=512, local_heads=4, local_kv_heads=2, local_head_dim=256,
                                 sliding_window=64, intermediate_size=1024, attn_implementation=impl)


@pytest.mark.parametrize("n", [300, 1024])
def test_decoder_logits_match_explicit_attention(n):
    register_triton_attention()
    ALL_ATTENTION_FUNCTIONS["explicit_test"] = explicit_attention
    torch.manual_seed(0)
    ours = Gemma4SyntheticDecoder(cfg("triton_gqa")).cuda().bfloat16().init_weights(seed=3)
    ref = Gemma4SyntheticDecoder(cfg("explicit_test")).cuda().bfloat16()
    ref.load_state_dict(ours.state_dict())
    ids = torch.randint(0, 2000, (2, n), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        a = ours(ids).float()
        b = ref(ids).float()
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    top1 = (a.argmax(-1) == b.argmax(-1)).float().mean().item()
    assert cos > 0.999, cos
    assert top1 > 0.98, top1


def test_decoder_backward_through_adapter():
    register_triton_attention()
    ALL_ATTENTION_FUNCTIONS["explicit_test"] = explicit_attention
    ours = Gemma4SyntheticDecoder(cfg("triton_gqa")).cuda().bfloat16().init_weights(seed=4)
    ref = Gemma4SyntheticDecoder(cfg("explicit_test")).cuda().bfloat16()
    ref.load_state_dict(ours.state_dict())
    ids = torch.randint(0, 2000, (1, 256), generator=torch.Generator().manual_seed(2)).cuda()
    for m in (ours, ref):
        loss = torch.nn.functional.cross_entropy(m(ids)[0, :-1].float(), ids[0, 1:])
        loss.backward()
    for (n1, p1), (_, p2) in zip(ours.named_parameters(), ref.named_parameters()):
        if p1.grad is None or p1.grad.abs().max() == 0:
            continue
        c = torch.nn.functional.cosine_similarity(p1.grad.float().flatten(), p2.grad.float().flatten(), dim=0).item()
        assert c > 0.99, (n1, c)
