"""``tutti.integration.vllm.green_context``: IO kernels on a green-context SM partition (tutti_b200's)."""
from tutti_b200.parallel.green_context import GreenIoStream, configured_io_sms, io_stream_on_sms  # noqa: F401
from tutti_b200.parallel.green_context import io_stream_on_sms as reserve_io_sms  # noqa: F401


def enabled() -> bool:
    return bool(configured_io_sms())
