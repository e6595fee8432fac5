"""A real vLLM engine driven through LMCacheB200ConnectorV1 on one GPU.

vLLM runs a tiny Llama with random ("dummy") weights and no tokenizer; its
own prefix cache is off.  The same 1000-token prompt is generated twice: the
first run stores the prompt KV through the connector, the second loads it
back into freshly allocated blocks.  Greedy outputs must match and the
engine counters must show the store and the retrieve.  vLLM keeps global
state, so the run happens in a child process."""

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, os, sys
os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
os.environ.setdefault("VLLM_ATTENTION_BACKEND", "FLASH_ATTN")
sys.path.insert(0, sys.argv[2])
from vllm import LLM, SamplingParams
from vllm.config import KVTransferConfig
from vllm.inputs import TokensPrompt

ktc = KVTransferConfig(
    kv_connector="LMCacheB200ConnectorV1",
    kv_connector_module_path="lmcache_ascend_b200.integration.vllm.connector",
    kv_role="kv_both",
    kv_connector_extra_config={"lmcache.chunk_size": 256,
                               "lmcache.max_local_cpu_size": 0.5})
llm = LLM(model=sys.argv[1], load_format="dummy", skip_tokenizer_init=True,
          enforce_eager=True, gpu_memory_utilization=0.2, max_model_len=2048,
          block_size=16, dtype="bfloat16", enable_prefix_caching=False,
          kv_transfer_config=ktc, seed=0)
sp = SamplingParams(max_tokens=8, temperature=0.0, detokenize=False)
prompt = [100 + (i * 7) % 3000 for i in range(1000)]
o1 = llm.generate([TokensPrompt(prompt_token_ids=prompt)], sp)
o2 = llm.generate([TokensPrompt(prompt_token_ids=prompt)], sp)
from lmcache_ascend_b200.utils.metrics import get_stats
c = get_stats().snapshot()["counters"]
print("RESULT " + json.dumps({"o1": list(o1[0].outputs[0].token_ids),
                              "o2": list(o2[0].outputs[0].token_ids),
                              "stored": c.get("stored_tokens", 0),
                              "retrieved": c.get("retrieved_tokens", 0)}), flush=True)
"""


def _model_dir(tmp_path):
    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama",
           "hidden_size": 256, "intermediate_size": 512, "num_attention_heads": 4,
           "num_key_value_heads": 2, "head_dim": 64, "num_hidden_layers": 2,
           "vocab_size": 4096, "max_position_embeddings": 4096, "rms_norm_eps": 1e-5,
           "rope_theta": 10000.0, "torch_dtype": "bfloat16", "tie_word_embeddings": False,
           "bos_token_id": 1, "eos_token_id": 2}
    d = tmp_path / "tiny-llama"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(cfg))
    return str(d)


def test_vllm_prefix_reuse_through_connector(tmp_path):
    pytest.importorskip("vllm")
    md = _model_dir(tmp_path)
    p = subprocess.run([sys.executable, "-c", CHILD, md, ROOT], capture_output=True,
                       text=True, timeout=900)
    lines = [l for l in p.stdout.splitlines() if l.startswith("RESULT ")]
    assert p.returncode == 0 and lines, (p.stdout[-3000:], p.stderr[-6000:])
    r = json.loads(lines[-1][len("RESULT "):])
    assert r["stored"] >= 1000, r
    assert r["retrieved"] >= 999, r
    assert r["o1"] == r["o2"], r
