//go:build !linux || !cgo || !cuda

// Package cuda without the B200 library: every entry point reports that
// the GPU is unavailable, as pkg/metal/metal_fallback.go does, and the
// engine takes its CPU branch.
package cuda

import (
	"errors"
	"unsafe"
)

var errUnsupported = errors.New("cuda: not built with the cuda tag on linux with cgo")

func Init() error                                       { return errUnsupported }
func IsAvailable() bool                                 { return false }
func BeginBatch()                                       {}
func EndBatch()                                         {}
func CreateBuffer(ptr unsafe.Pointer, size int) unsafe.Pointer { return nil }
func ReleaseBuffer(buf unsafe.Pointer)                  {}

func MatMulBuf(quantType int, y, x []float32, wBuf unsafe.Pointer, rows, cols int) error {
	return errUnsupported
}

func MatMulBatchBuf(quantType int, y, x []float32, wBuf unsafe.Pointer, batchSize, rows, cols int) error {
	return errUnsupported
}

func MatMulFusedGateUpBatchBuf(quantType int, y, x []float32, gateBuf, upBuf unsafe.Pointer,
	batchSize, rows, cols int) error {
	return errUnsupported
}

func MatMulQ8_0(y, x []float32, raw []byte, rows, cols int) error { return errUnsupported }
func MatMulQ4_K(y, x []float32, raw []byte, rows, cols int) error { return errUnsupported }
func MatMulQ6_K(y, x []float32, raw []byte, rows, cols int) error { return errUnsupported }
func AddResidual(x, proj []float32, dim int) error                 { return errUnsupported }
func SwiGLU(gate, up []float32, hiddenDim int) error               { return errUnsupported }

func FFN(x []float32, norm, gate, up, down unsafe.Pointer, dim, hidden int, eps float32) error {
	return errUnsupported
}

func ConnectTP(rank, world, maxDim int, allGather func([]byte) [][]byte) error { return errUnsupported }
func CloseTP() error                                                          { return errUnsupported }

func SetPDL(on bool) error         { return errUnsupported }
func SetQ6KMMA(on bool) error      { return errUnsupported }
func SetPrefillPair(on bool) error { return errUnsupported }
