from hilda_vllm_b200.engine.llm_engine import LLMEngine


class LLM(LLMEngine):
    pass
