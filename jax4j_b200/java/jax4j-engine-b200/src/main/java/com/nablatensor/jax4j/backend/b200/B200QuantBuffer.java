package com.nablatensor.jax4j.backend.b200;

import com.nablatensor.jax4j.tensor.DType;
import com.nablatensor.jax4j.tensor.Device;
import com.nablatensor.jax4j.tensor.QuantType;
import com.nablatensor.jax4j.tensor.Shape;
import com.nablatensor.jax4j.tensor.spi.DeviceBuffer;
import java.lang.foreign.MemorySegment;
import java.lang.ref.Cleaner;
import java.util.concurrent.atomic.AtomicBoolean;

/**
 * A quantized matrix held by the engine (j4b_qweight_t): GGUF blocks repacked on upload into
 * the engine's fragment layout (same byte count). {@link #dtype} is the logical (decoded) type,
 * F32, as for the reference's CpuQuantBuffer.
 */
final class B200QuantBuffer implements DeviceBuffer {
  private static final Cleaner CLEANER = Cleaner.create();

  private final MemorySegment handle;
  private final QuantType type;
  private final Shape shape;
  private final Device device;
  private final Free free;
  private final Cleaner.Cleanable cleanable;

  B200QuantBuffer(MemorySegment handle, QuantType type, Shape shape, Device device) {
    this.handle = handle;
    this.type = type;
    this.shape = shape;
    this.device = device;
    this.free = new Free(handle);
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

  QuantType type() {
    return type;
  }

  MemorySegment handle() {
    if (free.done.get()) throw new IllegalStateException("quantized buffer has been released");
    return handle;
  }

  void release() {
    cleanable.clean();
  }

  private static final class Free implements Runnable {
    private final MemorySegment handle;
    final AtomicBoolean done = new AtomicBoolean();

    Free(MemorySegment handle) {
      this.handle = handle;
    }

    @Override
    public void run() {
      if (done.compareAndSet(false, true)) B200Native.quantFree(handle);
    }
  }
}
