//go:build linux && cgo && cuda

// Package cuda is go-infer's GPU seam for the B200 library
// (include/goinfer_cuda.h, go-infer_b200/libgoinfer_cuda.so): the same Go API
// as pkg/metal (metal_darwin.go), so pkg/engine/weights.go switches its
// import and forward.go / engine.go stay as they are.  It is built only with
// the `cuda` tag on linux with cgo; cuda_fallback.go stubs it otherwise, as
// metal_fallback.go does for Metal.
//
// Calls are serialised inside the library (one mutex, one CUDA stream);
// outside BeginBatch/EndBatch each call copies its Go slices in and out
// before returning, so no Go pointer is kept after a call returns.  Inside a
// batch the output slices are written at EndBatch (the Metal contract).
package cuda

/*
#cgo CFLAGS: -I${SRCDIR}/../../../../include
#cgo LDFLAGS: -L${SRCDIR}/../../../../go-infer_b200 -lgoinfer_cuda -Wl,-rpath,${SRCDIR}/../../../../go-infer_b200
#include <stdlib.h>
#include "goinfer_cuda.h"
*/
import "C"

import (
	"bytes"
	"fmt"
	"os"
	"sync"
	"unsafe"
)

var (
	initOnce sync.Once
	initErr  error
)

func lastErr(what string, rc C.int) error {
	return fmt.Errorf("%s failed: %d (%s)", what, int(rc), C.GoString(C.gi_cuda_last_error()))
}

// Init mirrors metal.Init (metal_darwin.go:26).
func Init() error {
	initOnce.Do(func() {
		if rc := C.gi_cuda_init(); rc != 0 {
			initErr = lastErr("gi_cuda_init", rc)
		}
	})
	return initErr
}

// IsAvailable mirrors metal.IsAvailable (metal_darwin.go:37).
func IsAvailable() bool {
	if os.Getenv("DISABLE_CUDA") == "1" {
		return false
	}
	return bool(C.gi_cuda_is_available())
}

// BeginBatch / EndBatch mirror metal.BeginBatch / metal.EndBatch
// (metal_bridge.h:19-20): calls in between only enqueue; EndBatch waits and
// writes every output slice in call order.
func BeginBatch() { C.gi_cuda_begin_batch() }
func EndBatch()   { C.gi_cuda_end_batch() }

// CreateBuffer copies a tensor's raw GGUF bytes into device memory once
// (metal.CreateBuffer wraps unified memory instead); nil on failure.
func CreateBuffer(ptr unsafe.Pointer, size int) unsafe.Pointer {
	if ptr == nil || size == 0 {
		return nil
	}
	return unsafe.Pointer(C.gi_cuda_create_buffer(ptr, C.size_t(size)))
}

// ReleaseBuffer mirrors metal.ReleaseBuffer.
func ReleaseBuffer(buf unsafe.Pointer) {
	if buf != nil {
		C.gi_cuda_release_buffer(C.gi_cuda_buffer_t(buf))
	}
}

// MatMulBuf mirrors metal.MatMulBuf (metal_darwin.go:525): y = W x for the
// weight buffer of GGML type quantType.
func MatMulBuf(quantType int, y, x []float32, wBuf unsafe.Pointer, rows, cols int) error {
	if !IsAvailable() || len(y) < rows || len(x) < cols || wBuf == nil {
		return fmt.Errorf("cuda: unavailable or bad arguments")
	}
	rc := C.gi_cuda_gemv_buf(C.int(quantType), (*C.float)(&y[0]), (*C.float)(&x[0]),
		C.gi_cuda_buffer_t(wBuf), C.uint32_t(rows), C.uint32_t(cols))
	if rc != 0 {
		return lastErr("gi_cuda_gemv_buf", rc)
	}
	return nil
}

// MatMulBatchBuf mirrors metal.MatMulBatchBuf (metal_darwin.go:544):
// y[b*rows+r] = (W x_b)[r] for batchSize tokens.
func MatMulBatchBuf(quantType int, y, x []float32, wBuf unsafe.Pointer, batchSize, rows, cols int) error {
	if !IsAvailable() || len(y) < batchSize*rows || len(x) < batchSize*cols || wBuf == nil {
		return fmt.Errorf("cuda: unavailable or bad arguments")
	}
	rc := C.gi_cuda_gemm_buf(C.int(quantType), (*C.float)(&y[0]), (*C.float)(&x[0]),
		C.gi_cuda_buffer_t(wBuf), C.uint32_t(batchSize), C.uint32_t(rows), C.uint32_t(cols))
	if rc != 0 {
		return lastErr("gi_cuda_gemm_buf", rc)
	}
	return nil
}

// MatMulFusedGateUpBatchBuf mirrors metal.MatMulFusedGateUpBatchBuf
// (metal_darwin.go:564): y[b*rows+r] = silu(gate x_b)[r] * (up x_b)[r], Q4_K.
func MatMulFusedGateUpBatchBuf(quantType int, y, x []float32, gateBuf, upBuf unsafe.Pointer,
	batchSize, rows, cols int) error {
	if !IsAvailable() || len(y) < batchSize*rows || len(x) < batchSize*cols || gateBuf == nil || upBuf == nil {
		return fmt.Errorf("cuda: unavailable or bad arguments")
	}
	rc := C.gi_cuda_gemm_fused_gate_up_buf(C.int(quantType), (*C.float)(&y[0]), (*C.float)(&x[0]),
		C.gi_cuda_buffer_t(gateBuf), C.gi_cuda_buffer_t(upBuf), C.uint32_t(batchSize), C.uint32_t(rows),
		C.uint32_t(cols))
	if rc != 0 {
		return lastErr("gi_cuda_gemm_fused_gate_up_buf", rc)
	}
	return nil
}

func hostGemv(what string, fn func() C.int) error {
	if rc := fn(); rc != 0 {
		return lastErr(what, rc)
	}
	return nil
}

// MatMulQ8_0 / MatMulQ4_K / MatMulQ6_K mirror metal.MatMulQ8_0 / Q4_K / Q6_K
// (metal_darwin.go:800-860): host weights, copied to the device per call.
func MatMulQ8_0(y, x []float32, raw []byte, rows, cols int) error {
	return hostGemv("gi_cuda_gemv_q8_0", func() C.int {
		return C.gi_cuda_gemv_q8_0((*C.float)(&y[0]), (*C.float)(&x[0]), unsafe.Pointer(&raw[0]),
			C.uint32_t(rows), C.uint32_t(cols))
	})
}

func MatMulQ4_K(y, x []float32, raw []byte, rows, cols int) error {
	return hostGemv("gi_cuda_gemv_q4_k", func() C.int {
		return C.gi_cuda_gemv_q4_k((*C.float)(&y[0]), (*C.float)(&x[0]), unsafe.Pointer(&raw[0]),
			C.uint32_t(rows), C.uint32_t(cols))
	})
}

func MatMulQ6_K(y, x []float32, raw []byte, rows, cols int) error {
	return hostGemv("gi_cuda_gemv_q6_k", func() C.int {
		return C.gi_cuda_gemv_q6_k((*C.float)(&y[0]), (*C.float)(&x[0]), unsafe.Pointer(&raw[0]),
			C.uint32_t(rows), C.uint32_t(cols))
	})
}

// AddResidual mirrors metal.AddResidual (metal_darwin.go:743): x += proj.
func AddResidual(x, proj []float32, dim int) error {
	if rc := C.gi_cuda_add_residual((*C.float)(&x[0]), (*C.float)(&proj[0]), C.uint32_t(dim)); rc != 0 {
		return lastErr("gi_cuda_add_residual", rc)
	}
	return nil
}

// SwiGLU mirrors metal.SwiGLU (metal_darwin.go:730): gate = silu(gate) * up.
func SwiGLU(gate, up []float32, hiddenDim int) error {
	if rc := C.gi_cuda_swiglu((*C.float)(&gate[0]), (*C.float)(&up[0]), C.uint32_t(hiddenDim)); rc != 0 {
		return lastErr("gi_cuda_swiglu", rc)
	}
	return nil
}

// FFN runs the feed-forward half of a layer on this rank's shard (no
// single reference counterpart: forward.go:275-287's rmsnorm, gate/up
// MatMuls, SwiGLU, down MatMul and residual add): x += down(SwiGLU(gate(n),
// up(n))), n = RMSNorm(x) * norm.  After ConnectTP the down partials are
// summed across the ranks on the GPUs.
func FFN(x []float32, norm, gate, up, down unsafe.Pointer, dim, hidden int, eps float32) error {
	rc := C.gi_cuda_ffn_buf((*C.float)(&x[0]), C.gi_cuda_buffer_t(norm), C.gi_cuda_buffer_t(gate),
		C.gi_cuda_buffer_t(up), C.gi_cuda_buffer_t(down), C.uint32_t(dim), C.uint32_t(hidden), C.float(eps))
	if rc != 0 {
		return lastErr("gi_cuda_ffn_buf", rc)
	}
	return nil
}

// Config holds the model constants of pkg/engine/config.go that the decode
// entry points take.
type Config struct {
	NumLayers, Dim, HiddenDim, KVDim, VocabSize int
	NumHeads, NumKVHeads, HeadDim, MaxSeq        int
	NormEps, RopeTheta                           float32
}

// LayerWeights is metal_layer_weights_t's counterpart (metal_bridge.h:54-67):
// the buffer handles NewWeights creates (weights.go:35-38) and their types.
type LayerWeights = C.gi_cuda_layer_weights_t

// AllocBuffers mirrors metal.AllocBuffers (metal_bridge.h:23).
func AllocBuffers(c *Config) error {
	rc := C.gi_cuda_alloc_buffers(C.uint32_t(c.Dim), C.uint32_t(c.HiddenDim), C.uint32_t(c.KVDim),
		C.uint32_t(c.VocabSize), C.uint32_t(c.NumLayers), C.uint32_t(c.MaxSeq))
	if rc != 0 {
		return lastErr("gi_cuda_alloc_buffers", rc)
	}
	return nil
}

// ForwardTransformer mirrors metal.ForwardTransformer (forward.go:102-130,
// metal_bridge.h:134-157): x is the embedding of the current token; logits
// (len vocab) and the first-maximum token come back to the host.
func ForwardTransformer(x, logits []float32, layers []LayerWeights, outNorm, outW unsafe.Pointer, outType int,
	c *Config, pos, slot, active int, attnScale float32) (int, error) {
	var tok C.uint32_t
	rc := C.gi_cuda_forward_transformer((*C.float)(&x[0]), (*C.float)(&logits[0]), &tok,
		&layers[0], C.gi_cuda_buffer_t(outNorm), C.gi_cuda_buffer_t(outW), C.int(outType),
		C.uint32_t(c.NumLayers), C.uint32_t(c.Dim), C.uint32_t(c.HiddenDim), C.uint32_t(c.KVDim),
		C.uint32_t(c.VocabSize), C.uint32_t(c.NumHeads), C.uint32_t(c.NumKVHeads), C.uint32_t(c.HeadDim),
		C.uint32_t(pos), C.uint32_t(slot), C.uint32_t(c.MaxSeq), C.uint32_t(active),
		C.float(c.NormEps), C.float(c.RopeTheta), C.float(attnScale))
	if rc != 0 {
		return 0, lastErr("gi_cuda_forward_transformer", rc)
	}
	return int(tok), nil
}

// Model is the device-resident greedy loop (no reference counterpart: the
// engine's loop of engine.go:505-545 with the embedding lookup, argmax and
// position advance on the device, one CUDA-graph replay per token).
type Model struct {
	h      C.gi_cuda_model_t
	layers []LayerWeights // kept alive while the model exists
}

// NewModel builds the model over the weight buffers; tpWorld > 1 after
// ConnectTP with this rank's shards (rows of Q/K/V/gate/up/output, columns
// of O/down) and its vocabulary offset.
func NewModel(c *Config, layers []LayerWeights, tokEmbd unsafe.Pointer, tokType int, outNorm, outW unsafe.Pointer,
	outType, tpWorld, tpRank, vocabOffset int) (*Model, error) {
	m := &Model{layers: layers}
	d := (*C.gi_cuda_model_desc_t)(C.calloc(1, C.size_t(unsafe.Sizeof(C.gi_cuda_model_desc_t{}))))
	defer C.free(unsafe.Pointer(d))
	lay := (*LayerWeights)(C.calloc(C.size_t(len(layers)), C.size_t(unsafe.Sizeof(LayerWeights{}))))
	defer C.free(unsafe.Pointer(lay))
	copy(unsafe.Slice(lay, len(layers)), layers)
	d.num_layers, d.dim, d.hidden_dim = C.uint32_t(c.NumLayers), C.uint32_t(c.Dim), C.uint32_t(c.HiddenDim)
	d.num_heads, d.num_kv_heads, d.head_dim = C.uint32_t(c.NumHeads), C.uint32_t(c.NumKVHeads), C.uint32_t(c.HeadDim)
	d.vocab_size, d.max_seq = C.uint32_t(c.VocabSize), C.uint32_t(c.MaxSeq)
	d.norm_eps, d.rope_theta = C.float(c.NormEps), C.float(c.RopeTheta)
	d.layers = lay
	d.token_embd, d.token_embd_type = C.gi_cuda_buffer_t(tokEmbd), C.int(tokType)
	d.output_norm = C.gi_cuda_buffer_t(outNorm)
	d.output_weight, d.output_weight_type = C.gi_cuda_buffer_t(outW), C.int(outType)
	d.tp_world, d.tp_rank, d.vocab_offset = C.uint32_t(tpWorld), C.uint32_t(tpRank), C.uint32_t(vocabOffset)
	m.h = C.gi_cuda_model_create(d) // copies the descriptor and the layer table
	if m.h == nil {
		return nil, fmt.Errorf("gi_cuda_model_create failed (%s)", C.GoString(C.gi_cuda_last_error()))
	}
	return m, nil
}

// Close releases the model (not its weight buffers).
func (m *Model) Close() {
	if m.h != nil {
		C.gi_cuda_model_destroy(m.h)
		m.h = nil
	}
}

// Reset zeroes the KV cache.
func (m *Model) Reset() error {
	if rc := C.gi_cuda_model_reset(m.h); rc != 0 {
		return lastErr("gi_cuda_model_reset", rc)
	}
	return nil
}

// Generate runs the prompt and n greedy steps on the device
// (gi_cuda_model_generate); the ids come back once at the end.
func (m *Model) Generate(prompt []int32, startPos, n int) ([]uint32, error) {
	out := make([]uint32, n)
	rc := C.gi_cuda_model_generate(m.h, (*C.int32_t)(&prompt[0]), C.uint32_t(len(prompt)),
		C.uint32_t(startPos), C.uint32_t(n), (*C.uint32_t)(&out[0]), nil, nil)
	if rc != 0 {
		return nil, lastErr("gi_cuda_model_generate", rc)
	}
	return out, nil
}

// SetPersistent runs every layer of a step in one persistent kernel
// (gi_cuda_model_set_persistent; Q4_K layers without biases, -2 otherwise).
func (m *Model) SetPersistent(on bool) error {
	en := 0
	if on {
		en = 1
	}
	if rc := C.gi_cuda_model_set_persistent(m.h, C.int(en)); rc != 0 {
		return lastErr("gi_cuda_model_set_persistent", rc)
	}
	return nil
}

// ConnectTP is NewTPCoordinator's device half (tensor_parallel.go:13-31):
// after the existing handshake each rank publishes its 64-byte exchange-region
// handle (allGather returns every rank's, in rank order) and maps its peers'.
func ConnectTP(rank, world, maxDim int, allGather func([]byte) [][]byte) error {
	h := make([]byte, 64)
	if rc := C.gi_cuda_tp_prepare(C.int(world), C.uint32_t(maxDim), unsafe.Pointer(&h[0])); rc != 0 {
		return lastErr("gi_cuda_tp_prepare", rc)
	}
	all := bytes.Join(allGather(h), nil) // world * 64 bytes
	if rc := C.gi_cuda_tp_connect(C.int(rank), C.int(world), unsafe.Pointer(&all[0])); rc != 0 {
		return lastErr("gi_cuda_tp_connect", rc)
	}
	return nil
}

// CloseTP unmaps the peers (no model may use the exchange any more).
func CloseTP() error {
	if rc := C.gi_cuda_tp_close(); rc != 0 {
		return lastErr("gi_cuda_tp_close", rc)
	}
	return nil
}

// The launch switches of this library (no pkg/metal counterparts: each
// chooses between two ways this library runs the same arithmetic).
// SetPDL: programmatic dependent launch for stand-alone calls (off by
// default; the decode graphs always use it).  SetQ6KMMA: Q6_K GEMVs on the
// int8 tensor cores (on by default) or the CUDA cores.  SetPrefillPair:
// batched GEMMs on CTA pairs (off by default, slower on B200, bit-identical).
func SetPDL(on bool) error { return setSwitch("gi_cuda_set_pdl", C.gi_cuda_set_pdl(cBool(on))) }

func SetQ6KMMA(on bool) error {
	return setSwitch("gi_cuda_set_q6k_mma", C.gi_cuda_set_q6k_mma(cBool(on)))
}

func SetPrefillPair(on bool) error {
	return setSwitch("gi_cuda_set_prefill_pair", C.gi_cuda_set_prefill_pair(cBool(on)))
}

func cBool(on bool) C.int {
	if on {
		return 1
	}
	return 0
}

func setSwitch(what string, rc C.int) error {
	if rc != 0 {
		return lastErr(what, rc)
	}
	return nil
}
