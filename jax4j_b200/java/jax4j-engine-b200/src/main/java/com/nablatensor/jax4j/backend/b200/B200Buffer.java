package com.nablatensor.jax4j.backend.b200;

import com.nablatensor.jax4j.tensor.DType;
import com.nablatensor.jax4j.tensor.Device;
import com.nablatensor.jax4j.tensor.Shape;
import com.nablatensor.jax4j.tensor.spi.DeviceBuffer;
import java.lang.ref.Cleaner;
import java.util.concurrent.atomic.AtomicBoolean;

/**
 * A dense row-major f32 tensor in device memory: the device address (j4b_buf) from j4b_alloc and
 * its shape. Released explicitly through {@link B200Backend#release} (the Tensor.close contract,
 * idempotent) or, when unreachable, by a cleaner. j4b_free is stream-ordered on the device's
 * engine stream, so freeing never races a kernel that still reads the buffer.
 */
final class B200Buffer implements DeviceBuffer {
  private static final Cleaner CLEANER = Cleaner.create();

  private final long address;
  private final Shape shape;
  private final Device device;
  private final Free free;
  private final Cleaner.Cleanable cleanable;

  B200Buffer(long address, Shape shape, Device device) {
    this.address = address;
    this.shape = shape;
    this.device = device;
    this.free = new Free(address);
    this.cleanable = CLEANER.register(this, free);
  }

  @Override
  public Shape shape() {
    return shape;
  }

  @Override
  public DType dtype() {
    return DType.F32;
  }

  @Override
  public Device device() {
    return device;
  }

  long count() {
    return shape.size();
  }

  long bytes() {
    return Math.multiplyExact(shape.size(), 4L);
  }

  /** The device address; a released buffer is an error, as in the reference's CudaBuffer. */
  long address() {
    if (free.done.get()) throw new IllegalStateException("buffer has been released: " + shape);
    return address;
  }

  void release() {
    cleanable.clean();
  }

  /** Frees the address once; holds no reference to the buffer so the cleaner can run. */
  private static final class Free implements Runnable {
    private final long address;
    final AtomicBoolean done = new AtomicBoolean();

    Free(long address) {
      this.address = address;
    }

    @Override
    public void run() {
      if (done.compareAndSet(false, true)) B200Native.free(address);
    }
  }

  @Override
  public String toString() {
    return "B200Buffer" + shape + "@" + device;
  }
}
