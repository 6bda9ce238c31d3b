package com.nablatensor.jax4j.backend.b200;

import static com.nablatensor.jax4j.backend.b200.B200Native.I;
import static com.nablatensor.jax4j.backend.b200.B200Native.L;
import static com.nablatensor.jax4j.backend.b200.B200Native.P;
import static com.nablatensor.jax4j.backend.b200.B200Native.call;
import static com.nablatensor.jax4j.backend.b200.B200Native.sig;
import static java.lang.foreign.ValueLayout.ADDRESS;
import static java.lang.foreign.ValueLayout.JAVA_DOUBLE;
import static java.lang.foreign.ValueLayout.JAVA_INT;
import static java.lang.foreign.ValueLayout.JAVA_LONG;

import com.nablatensor.jax4j.engine.AadOptions;
import com.nablatensor.jax4j.engine.AadResult;
import com.nablatensor.jax4j.engine.AadTape;
import com.nablatensor.jax4j.engine.AbstractAadExecutable;
import java.lang.foreign.Arena;
import java.lang.foreign.MemoryLayout;
import java.lang.foreign.MemorySegment;

/**
 * A scalar-AAD tape compiled by one of the engine's three Monte-Carlo replay engines
 * (j4b_aad_compile): the generated per-tape kernel, the fixed interpreter, or one launch per node.
 * A replay of {@code paths} scenarios from {@code pathOffset} returns f64 sums of the output, its
 * square and each adjoint (j4b_aad_replay); the result is their mean and standard error, as the
 * reference's AadKernel / CudaInterpExecutable / CudaEagerExecutable report. Chunking and
 * calibration are the core's (AbstractAadExecutable.replaySafe / calibrate).
 */
final class B200AadExecutable extends AbstractAadExecutable {
  private static final MemoryLayout[] COMPILE = sig(I, I, I, P, P, P, P, I, P, I, I, I, L, P);
  private static final MemoryLayout[] REPLAY = sig(P, P, L, L, L, P, P);

  private final String engineName;
  private final MemorySegment handle;
  private final int channels;
  private final double compileSeconds;
  private boolean freed;

  private B200AadExecutable(AadTape tape, AadOptions options, String engineName, MemorySegment handle,
      int channels, double compileSeconds) {
    super(tape, options);
    this.engineName = engineName;
    this.handle = handle;
    this.channels = channels;
    this.compileSeconds = compileSeconds;
  }

  static B200AadExecutable compile(AadTape tape, AadOptions options, String engineName, int engine,
      long scratchOption) {
    int n = tape.size();
    int[] ops = new int[n], argA = new int[n], argB = new int[n];
    double[] constants = new double[n];
    for (int i = 0; i < n; i++) {
      ops[i] = tape.op(i).ordinal();
      argA[i] = tape.argA(i);
      argB[i] = tape.argB(i);
      constants[i] = tape.constant(i);
    }
    int[] inputNodes = new int[Math.max(1, tape.inputCount())];
    for (int j = 0; j < tape.inputCount(); j++) inputNodes[j] = tape.inputNode(j);
    int precision = options.precision() == AadOptions.Precision.FLOAT64 ? 8 : 4;
    try (Arena a = Arena.ofConfined()) {
      MemorySegment out = a.allocate(ADDRESS);
      call("j4b_aad_compile", COMPILE, 0, engine, n, a.allocateFrom(JAVA_INT, ops),
          a.allocateFrom(JAVA_INT, argA), a.allocateFrom(JAVA_INT, argB),
          a.allocateFrom(JAVA_DOUBLE, constants), tape.inputCount(),
          a.allocateFrom(JAVA_INT, inputNodes), tape.outputNode(), precision,
          options.adjoints() ? 1 : 0, scratchOption, out);
      MemorySegment handle = out.get(ADDRESS, 0);
      MemorySegment ch = a.allocate(JAVA_INT), secs = a.allocate(JAVA_DOUBLE), threads = a.allocate(JAVA_LONG);
      call("j4b_aad_info", sig(P, P, P, P), handle, ch, secs, threads);
      return new B200AadExecutable(tape, options, engineName, handle, ch.get(JAVA_INT, 0),
          secs.get(JAVA_DOUBLE, 0));
    }
  }

  @Override
  public String engineName() {
    return engineName;
  }

  @Override
  public double compileSeconds() {
    return compileSeconds;
  }

  @Override
  public synchronized AadResult replay(long paths, long pathOffset, long seed) {
    checkOpen();
    if (paths <= 0) throw new IllegalArgumentException("paths must be positive");
    double[] sums;
    long start = System.nanoTime();
    try (Arena a = Arena.ofConfined()) {
      MemorySegment in = a.allocateFrom(JAVA_DOUBLE, inputs.length == 0 ? new double[] {0} : inputs);
      MemorySegment out = a.allocate(JAVA_DOUBLE, channels);
      call("j4b_aad_replay", REPLAY, handle, in, paths, pathOffset, seed, out, MemorySegment.NULL);
      sums = out.toArray(JAVA_DOUBLE);
    }
    double seconds = (System.nanoTime() - start) * 1e-9;
    double mean = sums[0] / paths;
    double error = Double.NaN;
    if (paths > 1) {
      double variance = (sums[1] - paths * mean * mean) / (paths - 1);
      error = Math.sqrt(Math.max(0.0, variance) / paths);
    }
    double[] gradients = new double[tape.inputCount()];
    if (options.adjoints()) {
      for (int j = 0; j < gradients.length; j++) gradients[j] = sums[2 + j] / paths;
    }
    return new AadResult(mean, error, gradients, tape.inputNames(), paths, seconds);
  }

  @Override
  public synchronized void close() {
    super.close();
    if (!freed) {
      freed = true;
      call("j4b_aad_free", sig(P), handle);
    }
  }
}
