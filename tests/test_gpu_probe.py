"""The HBM-peak probe (``xcb_hbm_probe``; the reference's bulk-copy bandwidth probes are dead code in its shipped
file, kernels/moe_w4a16_h200/moe_w4a16.py:2890-3061) streams what it claims: its XOR checksum of every 32-bit word
read equals the checksum of the buffer, for the bulk-copy ring, the ring with the L2 evict-first hint and plain
vector loads."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,chunk,stages,ctas", [(0, 16384, 8, 1), (1, 32768, 6, 1), (2, 16, 1, 2)])
def test_probe_reads_every_byte(cuda_device, mode, chunk, stages, ctas):
    from xcalibur_b200 import _lib

    lib = _lib.load()
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    G = sms * ctas
    per = 16 * 32768                                     # bytes per CTA: a multiple of every chunk above
    g = torch.Generator(device=cuda_device).manual_seed(mode)
    raw = torch.randint(-2**31, 2**31 - 1, (G * per // 4 + 256,), generator=g, device=cuda_device,
                        dtype=torch.int32)
    skip = ((-raw.data_ptr()) % 1024) // 4                 # the probe wants a 1 KB aligned source
    buf = raw[skip:skip + G * per // 4]
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    sink = torch.zeros(1, dtype=torch.float32, device=cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    rc = lib.xcb_hbm_probe(buf.data_ptr(), G * per, mode, chunk, stages, ctas, 256, None, 0, status.data_ptr(),
                           sink.data_ptr(), stream)
    assert rc == _lib.XCB_OK
    torch.cuda.synchronize(cuda_device)
    assert int(status.item()) == 0
    want = np.bitwise_xor.reduce(buf.cpu().numpy().view(np.uint32))
    assert int(sink.view(torch.int32).cpu().numpy().view(np.uint32)[0]) == int(want)
