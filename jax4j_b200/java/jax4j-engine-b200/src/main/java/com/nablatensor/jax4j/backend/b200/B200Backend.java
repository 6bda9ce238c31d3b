package com.nablatensor.jax4j.backend.b200;

import static com.nablatensor.jax4j.backend.b200.B200Native.D;
import static com.nablatensor.jax4j.backend.b200.B200Native.F;
import static com.nablatensor.jax4j.backend.b200.B200Native.I;
import static com.nablatensor.jax4j.backend.b200.B200Native.L;
import static com.nablatensor.jax4j.backend.b200.B200Native.P;
import static com.nablatensor.jax4j.backend.b200.B200Native.call;
import static com.nablatensor.jax4j.backend.b200.B200Native.sig;
import static java.lang.foreign.ValueLayout.ADDRESS;
import static java.lang.foreign.ValueLayout.JAVA_FLOAT;
import static java.lang.foreign.ValueLayout.JAVA_INT;
import static java.lang.foreign.ValueLayout.JAVA_LONG;

import com.nablatensor.jax4j.tensor.ConvSpec;
import com.nablatensor.jax4j.tensor.DType;
import com.nablatensor.jax4j.tensor.Device;
import com.nablatensor.jax4j.tensor.DeviceType;
import com.nablatensor.jax4j.tensor.Op;
import com.nablatensor.jax4j.tensor.QuantType;
import com.nablatensor.jax4j.tensor.Shape;
import com.nablatensor.jax4j.tensor.expr.Expr;
import com.nablatensor.jax4j.tensor.spi.ComputeBackend;
import com.nablatensor.jax4j.tensor.spi.DeviceBuffer;
import com.nablatensor.jax4j.tensor.spi.QuantizedOps;
import java.lang.foreign.Arena;
import java.lang.foreign.MemoryLayout;
import java.lang.foreign.MemorySegment;
import java.util.ArrayList;
import java.util.Arrays;
import java.util.EnumSet;
import java.util.List;
import java.util.Map;
import java.util.Set;
import java.util.concurrent.ConcurrentHashMap;

/**
 * The B200 engine behind {@code -Djax4j.tensor.backend=cuda}: ComputeBackend
 * (jax4j-core tensor/spi/ComputeBackend.java) and QuantizedOps (tensor/spi/QuantizedOps.java) over
 * libjax4j_b200.so. Name "cuda" and device type CUDA, as the reference's CudaBackend
 * (jax4j-engine-cuda backend/cuda/CudaBackend.java:418-439), at priority 200 so that the registry
 * prefers it where both modules are on the class path.
 *
 * <p>Every operation is device-local (no host round trips): launches are asynchronous on the
 * engine's per-device stream, {@link #download} synchronises it. Shape checks raise the
 * reference's IllegalArgumentException before any launch. {@code fused} compiles each distinct
 * expression once into one sm_100a kernel (a one-call tape of j4b_tape_compile); matmul and conv
 * use the tcgen05 GEMM at fp32 accuracy unless {@code -Djax4j.b200.precision=1} selects bf16
 * operands.
 */
public final class B200Backend implements ComputeBackend, QuantizedOps {
  private static final MemorySegment ENGINE_STREAM = MemorySegment.NULL;
  private static final int PRECISION = Integer.getInteger("jax4j.b200.precision", 0);
  private static final Set<Integer> INITIALISED = ConcurrentHashMap.newKeySet();

  private static final MemoryLayout[] FILL = sig(L, L, F, P);
  private static final MemoryLayout[] BINARY = sig(I, L, L, L, L, P);
  private static final MemoryLayout[] SCALAR = sig(I, L, D, L, L, P);
  private static final MemoryLayout[] UNARY = sig(I, L, L, L, P);
  private static final MemoryLayout[] A_OUT_2D = sig(L, L, L, L, P);
  private static final MemoryLayout[] REDUCE = sig(L, L, L, P);
  private static final MemoryLayout[] AXIS = sig(L, L, L, L, L, P);
  private static final MemoryLayout[] AXIS_BACKWARD = sig(L, L, L, L, L, L, P);
  private static final MemoryLayout[] BROADCAST = sig(L, P, I, P, I, L, P);
  private static final MemoryLayout[] INDEX = sig(L, L, L, L, L, P);
  private static final MemoryLayout[] RELU_BACKWARD = sig(L, L, L, L, P);
  private static final MemoryLayout[] RANDOM = sig(L, L, L, L, P);
  private static final MemoryLayout[] MATMUL = sig(L, L, L, L, L, L, L, I, P);
  private static final MemoryLayout[] CONV = sig(L, L, L, L, I, I, I, I, I, I, I, I, P);
  private static final MemoryLayout[] COPY = sig(L, L, L, P);
  private static final MemoryLayout[] QMATVEC = sig(P, L, L, L, L, P);
  private static final MemoryLayout[] QGEMM = sig(P, L, L, L, I, P);
  private static final MemoryLayout[] QROW = sig(P, L, L, P);
  private static final MemoryLayout[] QUPLOAD = sig(I, P, L, I, L, L, P);
  private static final long TAPE_MAGIC = 0x314550415442344AL;

  /** Compiled fused expressions, keyed by postfix program and input shapes. */
  private final Map<String, FusedKernel> fusedKernels = new ConcurrentHashMap<>();

  @Override
  public String name() {
    return "cuda";
  }

  @Override
  public DeviceType deviceType() {
    return DeviceType.CUDA;
  }

  @Override
  public boolean isAvailable() {
    try {
      return B200Native.deviceCount() > 0;
    } catch (Throwable t) {
      return false;
    }
  }

  @Override
  public int priority() {
    return 200;
  }

  // ---- memory ----

  private static int deviceIndex(Device device) {
    if (device == null || device.type() != DeviceType.CUDA) {
      throw new IllegalArgumentException("B200 backend requires a CUDA device, got " + device);
    }
    int dev = device.index();
    if (INITIALISED.add(dev)) {
      try (Arena a = Arena.ofConfined()) {
        call("j4b_init", sig(P, I), a.allocateFrom(JAVA_INT, dev), 1);
      } catch (RuntimeException | Error e) {
        INITIALISED.remove(dev);
        throw e;
      }
    }
    return dev;
  }

  private static B200Buffer alloc(Shape shape, Device device) {
    int dev = deviceIndex(device);
    long bytes = Math.multiplyExact(shape.size(), 4L);
    try (Arena a = Arena.ofConfined()) {
      MemorySegment out = a.allocate(JAVA_LONG);
      call("j4b_alloc", sig(I, L, P), dev, bytes, out);
      return new B200Buffer(out.get(JAVA_LONG, 0), shape, device);
    }
  }

  private static B200Buffer b200(DeviceBuffer buffer) {
    if (buffer instanceof B200Buffer b) return b;
    throw new IllegalArgumentException("not a B200 device buffer: " + buffer);
  }

  private static B200QuantBuffer quant(DeviceBuffer buffer) {
    if (buffer instanceof B200QuantBuffer q) return q;
    throw new IllegalArgumentException("not a B200 quantized buffer: " + buffer);
  }

  @Override
  public DeviceBuffer upload(float[] data, Shape shape, DType dtype, Device device) {
    if (dtype != DType.F32) {
      throw new UnsupportedOperationException("CUDA float upload supports F32 only, got " + dtype);
    }
    if (data.length != shape.size()) {
      throw new IllegalArgumentException(data.length + " values do not fill " + shape);
    }
    B200Buffer out = alloc(shape, device);
    try (Arena a = Arena.ofConfined()) {
      MemorySegment host = a.allocateFrom(JAVA_FLOAT, data);
      call("j4b_h2d", sig(L, P, L, P), out.address(), host, out.bytes(), ENGINE_STREAM);
    }
    return out;
  }

  @Override
  public float[] download(DeviceBuffer buffer) {
    B200Buffer b = b200(buffer);
    try (Arena a = Arena.ofConfined()) {
      MemorySegment host = a.allocate(Math.max(4L, b.bytes()), 16);
      call("j4b_d2h", sig(P, L, L, P), host, b.address(), b.bytes(), ENGINE_STREAM);
      return host.asSlice(0, b.bytes()).toArray(JAVA_FLOAT);
    }
  }

  @Override
  public DeviceBuffer full(float value, Shape shape, DType dtype, Device device) {
    if (dtype != DType.F32) {
      throw new UnsupportedOperationException("CUDA fill supports F32 only, got " + dtype);
    }
    B200Buffer out = alloc(shape, device);
    call("j4b_fill", FILL, out.address(), out.count(), value, ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer randomUniform(long seed, long counter, Shape shape, Device device) {
    B200Buffer out = alloc(shape, device);
    call("j4b_random_uniform", RANDOM, seed, counter, out.address(), out.count(), ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer randomNormal(long seed, long counter, Shape shape, Device device) {
    B200Buffer out = alloc(shape, device);
    call("j4b_random_normal", RANDOM, seed, counter, out.address(), out.count(), ENGINE_STREAM);
    return out;
  }

  // ---- elementwise: Op ordinals are the engine's op codes (ADD 0 .. SIGN 15) ----

  @Override
  public DeviceBuffer binary(Op op, DeviceBuffer a, DeviceBuffer b) {
    B200Buffer left = b200(a), right = b200(b);
    if (left.count() != right.count()) {
      throw new IllegalArgumentException("shape mismatch: " + left.shape() + " vs " + right.shape());
    }
    B200Buffer out = alloc(left.shape(), left.device());
    call("j4b_binary", BINARY, op.ordinal(), left.address(), right.address(), out.address(),
        left.count(), ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer scalar(Op op, DeviceBuffer a, double value) {
    B200Buffer in = b200(a);
    B200Buffer out = alloc(in.shape(), in.device());
    call("j4b_scalar", SCALAR, op.ordinal(), in.address(), value, out.address(), in.count(),
        ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer unary(Op op, DeviceBuffer a) {
    B200Buffer in = b200(a);
    B200Buffer out = alloc(in.shape(), in.device());
    call("j4b_unary", UNARY, op.ordinal(), in.address(), out.address(), in.count(), ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer reluBackward(DeviceBuffer upstream, DeviceBuffer input) {
    B200Buffer up = b200(upstream), in = b200(input);
    if (up.count() != in.count()) {
      throw new IllegalArgumentException("shape mismatch: " + up.shape() + " vs " + in.shape());
    }
    B200Buffer out = alloc(up.shape(), up.device());
    call("j4b_relu_backward", RELU_BACKWARD, up.address(), in.address(), out.address(), up.count(),
        ENGINE_STREAM);
    return out;
  }

  /**
   * One sm_100a kernel per distinct expression (the reference's CudaJit compiles one NVRTC kernel
   * per fused call): the expression is serialised as the engine's postfix program
   * (0 idx | 1 op | 2 op | 3 op lo32 hi32) in a one-call tape, compiled once and replayed.
   */
  @Override
  public DeviceBuffer fused(Expr expr, DeviceBuffer[] inputs) {
    if (inputs.length == 0) throw new IllegalArgumentException("fused requires at least one input");
    B200Buffer[] in = new B200Buffer[inputs.length];
    for (int i = 0; i < inputs.length; i++) {
      in[i] = b200(inputs[i]);
      if (in[i].count() != in[0].count()) {
        throw new IllegalArgumentException("fused inputs must share element count");
      }
    }
    List<Long> program = new ArrayList<>();
    postfix(expr, program);
    StringBuilder key = new StringBuilder(program.toString());
    for (B200Buffer b : in) key.append(Arrays.toString(b.shape().dims()));
    int dev = deviceIndex(in[0].device());
    key.append('@').append(dev);
    FusedKernel kernel = fusedKernels.computeIfAbsent(key.toString(),
        k -> FusedKernel.compile(dev, in, program));
    B200Buffer out = alloc(in[0].shape(), in[0].device());
    kernel.launch(in, out);
    return out;
  }

  private static void postfix(Expr expr, List<Long> out) {
    switch (expr) {
      case Expr.Input x -> {
        out.add(0L);
        out.add((long) x.index());
      }
      case Expr.Unary u -> {
        postfix(u.in(), out);
        out.add(1L);
        out.add((long) u.op().ordinal());
      }
      case Expr.Binary b -> {
        postfix(b.left(), out);
        postfix(b.right(), out);
        out.add(2L);
        out.add((long) b.op().ordinal());
      }
      case Expr.Scalar s -> {
        postfix(s.in(), out);
        long bits = Double.doubleToRawLongBits(s.value());
        out.add(3L);
        out.add((long) s.op().ordinal());
        out.add((long) (int) bits);
        out.add((long) (int) (bits >>> 32));
      }
    }
  }

  /** A compiled one-call tape (j4b_tape_t); launches of one tape are serialised. */
  private static final class FusedKernel {
    private final MemorySegment tape;

    private FusedKernel(MemorySegment tape) {
      this.tape = tape;
    }

    static FusedKernel compile(int dev, B200Buffer[] in, List<Long> program) {
      List<Long> w = new ArrayList<>();
      int n = in.length;
      // header; buffer shapes: the n inputs, then the output (shaped as input 0)
      w.addAll(List.of(TAPE_MAGIC, (long) n + 1, (long) n, 1L, 1L));
      for (int i = 0; i <= n; i++) {
        int[] dims = in[i == n ? 0 : i].shape().dims();
        w.add((long) dims.length);
        for (int d : dims) w.add((long) d);
      }
      for (int i = 0; i < n; i++) w.add((long) i);
      w.add((long) n);
      w.addAll(List.of(2L, (long) n, (long) n));
      for (int i = 0; i < n; i++) w.add((long) i);
      w.add((long) program.size());
      w.addAll(program);
      long[] words = w.stream().mapToLong(Long::longValue).toArray();
      try (Arena a = Arena.ofConfined()) {
        MemorySegment out = a.allocate(ADDRESS);
        call("j4b_tape_compile", sig(I, P, L, P), dev, a.allocateFrom(JAVA_LONG, words),
            (long) words.length, out);
        return new FusedKernel(out.get(ADDRESS, 0));
      }
    }

    synchronized void launch(B200Buffer[] in, B200Buffer out) {
      try (Arena a = Arena.ofConfined()) {
        long[] ins = new long[in.length];
        for (int i = 0; i < in.length; i++) ins[i] = in[i].address();
        call("j4b_tape_launch", sig(P, P, I, P, I, P), tape, a.allocateFrom(JAVA_LONG, ins),
            in.length, a.allocateFrom(JAVA_LONG, out.address()), 1, ENGINE_STREAM);
      }
    }
  }

  // ---- movement and contraction ----

  @Override
  public DeviceBuffer transpose(DeviceBuffer a) {
    B200Buffer in = b200(a);
    if (in.shape().rank() != 2) {
      throw new IllegalArgumentException("transpose requires a rank-2 tensor, got " + in.shape());
    }
    int r = in.shape().dim(0), c = in.shape().dim(1);
    B200Buffer out = alloc(Shape.of(c, r), in.device());
    call("j4b_transpose", A_OUT_2D, in.address(), out.address(), (long) r, (long) c, ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer matmul(DeviceBuffer a, DeviceBuffer b) {
    B200Buffer left = b200(a), right = b200(b);
    Shape sa = left.shape(), sb = right.shape();
    if (sa.rank() != 2 || sb.rank() != 2 || sa.dim(1) != sb.dim(0)) {
      throw new IllegalArgumentException("incompatible matmul shapes: " + sa + " x " + sb);
    }
    int m = sa.dim(0), k = sa.dim(1), n = sb.dim(1);
    B200Buffer out = alloc(Shape.of(m, n), left.device());
    call("j4b_matmul", MATMUL, left.address(), right.address(), out.address(), 1L, (long) m,
        (long) k, (long) n, PRECISION, ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer batchedMatmul(DeviceBuffer a, DeviceBuffer b) {
    B200Buffer left = b200(a), right = b200(b);
    Shape sa = left.shape(), sb = right.shape();
    if (sa.rank() != 3 || sb.rank() != 3 || sa.dim(0) != sb.dim(0) || sa.dim(2) != sb.dim(1)) {
      throw new IllegalArgumentException("incompatible batched matmul shapes: " + sa + " x " + sb);
    }
    int batch = sa.dim(0), m = sa.dim(1), k = sa.dim(2), n = sb.dim(2);
    B200Buffer out = alloc(Shape.of(batch, m, n), left.device());
    call("j4b_matmul", MATMUL, left.address(), right.address(), out.address(), (long) batch,
        (long) m, (long) k, (long) n, PRECISION, ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer sliceAxis0(DeviceBuffer input, int index) {
    B200Buffer in = b200(input);
    Shape shape = in.shape();
    if (shape.rank() < 1 || index < 0 || index >= shape.dim(0)) {
      throw new IllegalArgumentException("axis-0 index " + index + " is out of bounds for " + shape);
    }
    long slice = shape.size() / shape.dim(0);
    B200Buffer out = alloc(Shape.of(Arrays.copyOfRange(shape.dims(), 1, shape.rank())), in.device());
    call("j4b_d2d", COPY, out.address(), in.address() + 4L * index * slice, 4L * slice,
        ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer stackAxis0(DeviceBuffer[] inputs) {
    if (inputs.length == 0) {
      throw new IllegalArgumentException("stackAxis0 requires at least one input");
    }
    B200Buffer first = b200(inputs[0]);
    for (DeviceBuffer input : inputs) {
      if (!input.shape().equals(first.shape()) || input.dtype() != first.dtype()
          || !input.device().equals(first.device())) {
        throw new IllegalArgumentException(
            "stackAxis0 inputs must have identical shape, dtype, and device");
      }
    }
    int[] dims = first.shape().dims();
    int[] outDims = new int[dims.length + 1];
    outDims[0] = inputs.length;
    System.arraycopy(dims, 0, outDims, 1, dims.length);
    B200Buffer out = alloc(Shape.of(outDims), first.device());
    for (int i = 0; i < inputs.length; i++) {
      call("j4b_d2d", COPY, out.address() + (long) i * first.bytes(), b200(inputs[i]).address(),
          first.bytes(), ENGINE_STREAM);
    }
    return out;
  }

  @Override
  public DeviceBuffer reshape(DeviceBuffer a, Shape target) {
    B200Buffer in = b200(a);
    if (target.size() != in.count()) {
      throw new IllegalArgumentException("cannot reshape " + in.shape() + " to " + target);
    }
    B200Buffer out = alloc(target, in.device());
    call("j4b_d2d", COPY, out.address(), in.address(), in.bytes(), ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer broadcastTo(DeviceBuffer a, Shape target) {
    B200Buffer in = b200(a);
    if (in.shape().equals(target)) return in;
    if (!Shape.broadcast(in.shape(), target).equals(target)) {
      throw new IllegalArgumentException("cannot broadcast shape " + in.shape() + " to " + target);
    }
    B200Buffer out = alloc(target, in.device());
    try (Arena ar = Arena.ofConfined()) {
      long[] src = Arrays.stream(in.shape().dims()).asLongStream().toArray();
      long[] dst = Arrays.stream(target.dims()).asLongStream().toArray();
      MemorySegment s = ar.allocateFrom(JAVA_LONG, src.length == 0 ? new long[] {1} : src);
      call("j4b_broadcast_to", BROADCAST, in.address(), s, src.length,
          ar.allocateFrom(JAVA_LONG, dst), dst.length, out.address(), ENGINE_STREAM);
    }
    return out;
  }

  /** The index map as a device int32 buffer, range-checked on the host first (-1 = zero). */
  private static B200Buffer indexMap(int[] indices, long bound, Device device) {
    for (int index : indices) {
      if (index < -1 || index >= bound) throw new IllegalArgumentException("index out of bounds");
    }
    B200Buffer map = alloc(Shape.of(Math.max(1, indices.length)), device);
    try (Arena a = Arena.ofConfined()) {
      call("j4b_h2d", sig(L, P, L, P), map.address(), a.allocateFrom(JAVA_INT, indices),
          4L * indices.length, ENGINE_STREAM);
    }
    return map;
  }

  @Override
  public DeviceBuffer reindex(DeviceBuffer input, Shape target, int[] indices) {
    if (indices.length != target.size()) throw new IllegalArgumentException("index map size");
    B200Buffer in = b200(input);
    B200Buffer map = indexMap(indices, in.count(), in.device());
    B200Buffer out = alloc(target, in.device());
    call("j4b_reindex", INDEX, in.address(), in.count(), map.address(), out.count(), out.address(),
        ENGINE_STREAM);
    map.release();
    return out;
  }

  @Override
  public DeviceBuffer scatterAdd(DeviceBuffer input, Shape target, int[] indices) {
    B200Buffer in = b200(input);
    if (indices.length != in.count()) throw new IllegalArgumentException("index map size");
    B200Buffer map = indexMap(indices, target.size(), in.device());
    B200Buffer out = alloc(target, in.device());
    call("j4b_scatter_add", INDEX, in.address(), in.count(), map.address(), target.size(),
        out.address(), ENGINE_STREAM);
    map.release();
    return out;
  }

  // ---- reductions ----

  @Override
  public DeviceBuffer reduceSum(DeviceBuffer a) {
    B200Buffer in = b200(a);
    B200Buffer out = alloc(Shape.of(1), in.device());
    call("j4b_reduce_sum", REDUCE, in.address(), in.count(), out.address(), ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer reduceMax(DeviceBuffer a) {
    B200Buffer in = b200(a);
    B200Buffer out = alloc(Shape.of(1), in.device());
    call("j4b_reduce_max", REDUCE, in.address(), in.count(), out.address(), ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer sumAxis0(DeviceBuffer a) {
    if (a.shape().rank() != 2) {
      throw new IllegalStateException("sumAxis0 requires a rank-2 tensor, got " + a.shape());
    }
    return sumAxis(a, 0, false);
  }

  /** (outer, axis, inner) extents of a reduction over {@code axis}. */
  private static long[] split(Shape shape, int axis) {
    if (axis < 0 || axis >= shape.rank()) {
      throw new IllegalArgumentException("axis " + axis + " is out of bounds for shape " + shape);
    }
    long outer = 1, inner = 1;
    for (int i = 0; i < axis; i++) outer *= shape.dim(i);
    for (int i = axis + 1; i < shape.rank(); i++) inner *= shape.dim(i);
    return new long[] {outer, shape.dim(axis), inner};
  }

  private static Shape reduced(Shape shape, int axis, boolean keepDims) {
    int[] dims = shape.dims();
    if (keepDims) {
      int[] kept = dims.clone();
      kept[axis] = 1;
      return Shape.of(kept);
    }
    int[] out = new int[dims.length - 1];
    for (int i = 0, j = 0; i < dims.length; i++) if (i != axis) out[j++] = dims[i];
    return Shape.of(out);
  }

  private DeviceBuffer axisReduce(String entry, DeviceBuffer a, int axis, boolean keepDims) {
    B200Buffer in = b200(a);
    long[] s = split(in.shape(), axis);
    B200Buffer out = alloc(reduced(in.shape(), axis, keepDims), in.device());
    call(entry, AXIS, in.address(), s[0], s[1], s[2], out.address(), ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer sumAxis(DeviceBuffer a, int axis, boolean keepDims) {
    return axisReduce("j4b_sum_axis", a, axis, keepDims);
  }

  @Override
  public DeviceBuffer maxAxis(DeviceBuffer a, int axis, boolean keepDims) {
    return axisReduce("j4b_max_axis", a, axis, keepDims);
  }

  @Override
  public DeviceBuffer argMaxAxis(DeviceBuffer a, int axis) {
    return axisReduce("j4b_argmax_axis", a, axis, false);
  }

  @Override
  public DeviceBuffer maxAxisBackward(DeviceBuffer upstream, DeviceBuffer input, int axis) {
    B200Buffer up = b200(upstream), in = b200(input);
    long[] s = split(in.shape(), axis);
    if (up.count() != s[0] * s[2]) {
      throw new IllegalArgumentException("maxAxisBackward gradient shape " + up.shape()
          + " is incompatible with input " + in.shape() + " and axis " + axis);
    }
    B200Buffer out = alloc(in.shape(), in.device());
    call("j4b_max_axis_backward", AXIS_BACKWARD, up.address(), in.address(), s[0], s[1], s[2],
        out.address(), ENGINE_STREAM);
    return out;
  }

  // ---- convolution: im2col + tcgen05 GEMM; gradients by gather col2im ----

  private DeviceBuffer conv(String entry, B200Buffer a, B200Buffer b, ConvSpec spec, Shape outShape) {
    B200Buffer out = alloc(outShape, a.device());
    call(entry, CONV, a.address(), b.address(), out.address(), (long) a.shape().dim(0),
        spec.inChannels(), spec.inHeight(), spec.inWidth(), spec.outChannels(), spec.kernel(),
        spec.stride(), spec.pad(), PRECISION, ENGINE_STREAM);
    return out;
  }

  private static int batchOf(B200Buffer x, int rowSize, String what, ConvSpec spec) {
    if (x.shape().rank() != 2 || x.shape().dim(1) != rowSize) {
      throw new IllegalArgumentException(what + " shape " + x.shape() + " does not match " + spec);
    }
    return x.shape().dim(0);
  }

  @Override
  public DeviceBuffer conv2d(DeviceBuffer x, DeviceBuffer w, ConvSpec spec) {
    B200Buffer in = b200(x), filters = b200(w);
    int batch = batchOf(in, spec.inputSize(), "conv2d input", spec);
    if (!filters.shape().equals(spec.weightShape())) {
      throw new IllegalArgumentException("conv2d weight shape " + filters.shape() + " does not match " + spec);
    }
    return conv("j4b_conv2d", in, filters, spec, spec.outputShape(batch));
  }

  @Override
  public DeviceBuffer conv2dGradInput(DeviceBuffer upstream, DeviceBuffer w, ConvSpec spec) {
    B200Buffer up = b200(upstream), filters = b200(w);
    int batch = batchOf(up, spec.outputSize(), "conv2dGradInput upstream", spec);
    if (!filters.shape().equals(spec.weightShape())) {
      throw new IllegalArgumentException("conv2dGradInput weight shape " + filters.shape()
          + " does not match " + spec);
    }
    return conv("j4b_conv2d_grad_input", up, filters, spec, spec.inputShape(batch));
  }

  @Override
  public DeviceBuffer conv2dGradWeight(DeviceBuffer x, DeviceBuffer upstream, ConvSpec spec) {
    B200Buffer in = b200(x), up = b200(upstream);
    int batch = batchOf(in, spec.inputSize(), "conv2dGradWeight input", spec);
    if (!up.shape().equals(spec.outputShape(batch))) {
      throw new IllegalArgumentException("conv2dGradWeight upstream shape " + up.shape()
          + " does not match " + spec);
    }
    return conv("j4b_conv2d_grad_weight", in, up, spec, spec.weightShape());
  }

  // ---- lifecycle ----

  @Override
  public void sync() {
    for (int dev : INITIALISED) call("j4b_sync", sig(I), dev);
  }

  /** Idempotent, as Tensor.close requires; quantized buffers are released the same way. */
  @Override
  public void release(DeviceBuffer buffer) {
    if (buffer instanceof B200Buffer b) b.release();
    else if (buffer instanceof B200QuantBuffer q) q.release();
  }

  // ---- QuantizedOps: GGUF blocks dequantised inside the GEMV ----

  @Override
  public Set<QuantType> supportedQuantTypes() {
    try (Arena a = Arena.ofConfined()) {
      MemorySegment ids = a.allocate(JAVA_INT, 16), n = a.allocate(JAVA_INT);
      call("j4b_quant_supported", sig(P, I, P), ids, 16, n);
      Set<QuantType> out = EnumSet.noneOf(QuantType.class);
      for (int i = 0; i < n.get(JAVA_INT, 0); i++) out.add(QuantType.byId(ids.getAtIndex(JAVA_INT, i)));
      return out;
    }
  }

  @Override
  public DeviceBuffer uploadQuantized(MemorySegment blocks, QuantType type, Shape logicalShape,
      Device device) {
    if (logicalShape.rank() != 2) {
      throw new IllegalArgumentException("quantized matrices are rank 2, got " + logicalShape);
    }
    int dev = deviceIndex(device);
    try (Arena a = Arena.ofConfined()) {
      MemorySegment src = blocks;
      if (!blocks.isNative()) {
        src = a.allocate(blocks.byteSize(), 16);
        MemorySegment.copy(blocks, 0, src, 0, blocks.byteSize());
      }
      MemorySegment out = a.allocate(ADDRESS);
      call("j4b_quant_upload", QUPLOAD, dev, src, src.byteSize(), type.id(),
          (long) logicalShape.dim(0), (long) logicalShape.dim(1), out);
      return new B200QuantBuffer(out.get(ADDRESS, 0), type, logicalShape, device);
    }
  }

  /** y = W x; x of shape (cols) is the reference call, (batch, cols) decodes a batch at once. */
  @Override
  public DeviceBuffer quantMatvec(DeviceBuffer weights, DeviceBuffer x) {
    return matvec(quant(weights), b200(x), null);
  }

  @Override
  public DeviceBuffer quantMatvecAdd(DeviceBuffer weights, DeviceBuffer x, DeviceBuffer add) {
    return matvec(quant(weights), b200(x), b200(add));
  }

  private DeviceBuffer matvec(B200QuantBuffer w, B200Buffer x, B200Buffer add) {
    int rows = w.shape().dim(0), cols = w.shape().dim(1);
    Shape xs = x.shape();
    if (xs.rank() < 1 || xs.rank() > 2 || xs.dim(xs.rank() - 1) != cols) {
      throw new IllegalArgumentException("quantMatvec shape mismatch: " + w.shape() + " x " + xs);
    }
    int batch = xs.rank() == 1 ? 1 : xs.dim(0);
    Shape outShape = xs.rank() == 1 ? Shape.of(rows) : Shape.of(batch, rows);
    if (add != null && add.count() != (long) batch * rows) {
      throw new IllegalArgumentException("quantMatvecAdd addend shape " + add.shape()
          + " does not match " + outShape);
    }
    B200Buffer out = alloc(outShape, x.device());
    call("j4b_quant_matvec", QMATVEC, w.handle(), x.address(), add == null ? 0L : add.address(),
        out.address(), (long) batch, ENGINE_STREAM);
    return out;
  }

  /**
   * Prefill projection y [m, rows] = x [m, cols] . W^T on the tcgen05 tensor cores (no
   * QuantizedOps counterpart: the reference has only the rank-1 quantMatvec). precision 1 = bf16
   * operands, 0 = fp32-accurate split.
   */
  public DeviceBuffer quantMatmul(DeviceBuffer weights, DeviceBuffer x, int precision) {
    B200QuantBuffer w = quant(weights);
    B200Buffer in = b200(x);
    if (in.shape().rank() != 2 || in.shape().dim(1) != w.shape().dim(1)) {
      throw new IllegalArgumentException("quantMatmul shape mismatch: " + w.shape() + " x " + in.shape());
    }
    B200Buffer out = alloc(Shape.of(in.shape().dim(0), w.shape().dim(0)), in.device());
    call("j4b_quant_gemm", QGEMM, w.handle(), in.address(), out.address(),
        (long) in.shape().dim(0), precision, ENGINE_STREAM);
    return out;
  }

  @Override
  public DeviceBuffer quantGatherRow(DeviceBuffer weights, int row) {
    B200QuantBuffer w = quant(weights);
    if (w.shape().rank() != 2) {
      throw new IllegalArgumentException(
          "quantGatherRow requires a rank-2 quantized matrix, got " + w.shape());
    }
    B200Buffer out = alloc(Shape.of(w.shape().dim(1)), w.device());
    call("j4b_quant_gather_row", QROW, w.handle(), (long) row, out.address(), ENGINE_STREAM);
    return out;
  }
}
