"""``python -m kvbm.vllm`` starts the prefill server (``kvbm.vllm.prefill``)."""

from kvbm.vllm.prefill import main

if __name__ == "__main__":
    main()
