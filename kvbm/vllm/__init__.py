"""vLLM integration (``kv_connector_module_path=kvbm.vllm.connector``)."""
