package com.nablatensor.jax4j.backend.b200;

import static com.nablatensor.jax4j.backend.b200.B200Native.I;
import static com.nablatensor.jax4j.backend.b200.B200Native.L;
import static com.nablatensor.jax4j.backend.b200.B200Native.P;
import static com.nablatensor.jax4j.backend.b200.B200Native.call;
import static com.nablatensor.jax4j.backend.b200.B200Native.sig;

import com.nablatensor.jax4j.engine.AadEngine;
import com.nablatensor.jax4j.engine.AadExecutable;
import com.nablatensor.jax4j.engine.AadOptions;
import com.nablatensor.jax4j.engine.AadTape;
import java.lang.foreign.Arena;
import java.lang.foreign.MemorySegment;

/**
 * The engine's three scalar-AAD replay engines as AadEngine providers, named as the reference's
 * CUDA engines (jax4j-engine-cuda engine/CudaAadEngine.java, CudaInterpEngine.java,
 * CudaEagerEngine.java) and ranked one above each, so that {@code -Dnablatensor.engine=cuda}
 * (AadEngines.find takes the highest priority of a name) selects the B200 engine where both
 * modules are on the class path. Like the reference's, they decline randu() and named streams
 * (AadEngine.requireBasicRandom) and multi-output tapes (requireSingleOutput).
 */
final class B200AadEngines {
  private B200AadEngines() {}

  static final int GENERATED = 0, INTERP = 1, EAGER = 2;

  abstract static class Base implements AadEngine {
    private final String name;
    private final int priority;
    private final int engine;
    private final String optionKey;

    Base(String name, int priority, int engine, String optionKey) {
      this.name = name;
      this.priority = priority;
      this.engine = engine;
      this.optionKey = optionKey;
    }

    @Override
    public String name() {
      return name;
    }

    @Override
    public int priority() {
      return priority;
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
    public boolean supports(AadOptions options) {
      return true;
    }

    @Override
    public String describe() {
      try (Arena a = Arena.ofConfined()) {
        MemorySegment buf = a.allocate(256);
        call("j4b_device_name", sig(I, P, L), 0, buf, 256L);
        return "B200 · " + buf.getString(0) + " · sm_100a";
      } catch (Throwable t) {
        return "B200 · no device";
      }
    }

    @Override
    public AadExecutable compile(AadTape tape, AadOptions options) {
      AadEngine.requireBasicRandom(tape, name);
      AadEngine.requireSingleOutput(tape, name);
      long scratch = 0;
      if (optionKey != null) {
        String v = options.engineOptions(name).get(optionKey);
        if (v != null) scratch = Long.parseLong(v.trim());
      }
      return B200AadExecutable.compile(tape, options, name, engine, scratch);
    }
  }
}
